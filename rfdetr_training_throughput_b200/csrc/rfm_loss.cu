// Matched-box losses of the DETR-family criterion (SetCriterion.loss_boxes),
// fed directly by the packed pairs rfm_lsap writes.
//
// The reference path feeds the criterion index tensors: the criterion gathers
// the matched prediction boxes (outputs["pred_boxes"][idx], criterion.py:904/906
// as cited at patches.py:339-341) and the matched target boxes, takes the L1 of
// their cxcywh coordinates and the diagonal of an N x N generalized-IoU matrix.
// Here one kernel reads each matched (query, target) pair where the solver put
// it, evaluates both terms for the pair, and reduces per (layer, image) in a
// fixed order (deterministic); the backward kernel writes the pair's gradient
// straight into its prediction box's slot (every (layer, image, query) is
// matched at most once, so there are no write conflicts).
//
// Per pair, with p = pred box (cx, cy, w, h), t = target box, xyxy corners:
//   l1   = |p.cx - t.cx| + |p.cy - t.cy| + |p.w - t.w| + |p.h - t.h|
//   giou = iou - (hull - union) / hull,   iou = inter / union,
//   inter = clamp(min(x1) - max(x0), 0) * clamp(min(y1) - max(y0), 0),
//   union = area_p + area_t - inter, hull = clamp(max(x1) - min(x0), 0) * (same in y)
// and the loss terms summed per layer are l1 and 1 - giou.  Gradients follow
// torch's autograd of that expression: min/max split ties evenly between their
// operands, clamp(min=0) passes the gradient at 0, |x| has slope sign(x).
#include "rfm_common.cuh"

namespace rfm {
namespace {

constexpr int kLossThreads = 128;

struct LossArgs {
  const float4* pred;           // [L, B, Q] cxcywh
  const float4* tgt;            // [S] cxcywh
  const int32_t* tgt_offsets;   // [B + 1]
  const int64_t* query_idx;     // [total]
  const int64_t* target_idx;    // [total]
  const int32_t* pair_offsets;  // [L * B + 1]
  int L, B, Q, S;
  float* l1_part;               // [L * B]
  float* giou_part;             // [L * B]
  const float* grad_l1;         // [L]
  const float* grad_giou;       // [L]
  float4* grad_pred;            // [L, B, Q]
};

struct Xyxy {
  float x0, y0, x1, y1;
};

__device__ __forceinline__ Xyxy xyxy(float4 b) {
  const float hw = __fmul_rn(0.5f, b.z);
  const float hh = __fmul_rn(0.5f, b.w);
  return Xyxy{__fsub_rn(b.x, hw), __fsub_rn(b.y, hh), __fadd_rn(b.x, hw), __fadd_rn(b.y, hh)};
}

struct GiouTerms {
  float iw, ih, iwc, ihc, inter, area_p, uni, ew, eh, ewc, ehc, hull, giou;
};

__device__ __forceinline__ GiouTerms giou_terms(const Xyxy& p, const Xyxy& t) {
  GiouTerms g;
  const float area_t = __fmul_rn(__fsub_rn(t.x1, t.x0), __fsub_rn(t.y1, t.y0));
  g.area_p = __fmul_rn(__fsub_rn(p.x1, p.x0), __fsub_rn(p.y1, p.y0));
  g.iw = __fsub_rn(fminf(p.x1, t.x1), fmaxf(p.x0, t.x0));
  g.ih = __fsub_rn(fminf(p.y1, t.y1), fmaxf(p.y0, t.y0));
  g.iwc = fmaxf(g.iw, 0.0f);
  g.ihc = fmaxf(g.ih, 0.0f);
  g.inter = __fmul_rn(g.iwc, g.ihc);
  g.uni = __fsub_rn(__fadd_rn(g.area_p, area_t), g.inter);
  g.ew = __fsub_rn(fmaxf(p.x1, t.x1), fminf(p.x0, t.x0));
  g.eh = __fsub_rn(fmaxf(p.y1, t.y1), fminf(p.y0, t.y0));
  g.ewc = fmaxf(g.ew, 0.0f);
  g.ehc = fmaxf(g.eh, 0.0f);
  g.hull = __fmul_rn(g.ewc, g.ehc);
  const float iou = __fdiv_rn(g.inter, g.uni);
  g.giou = __fsub_rn(iou, __fdiv_rn(__fsub_rn(g.hull, g.uni), g.hull));
  return g;
}

// d max(a, b) / d a with torch's even split of ties; d min(a, b) / d a likewise.
__device__ __forceinline__ float dmax_a(float a, float b) { return a > b ? 1.0f : (a == b ? 0.5f : 0.0f); }
__device__ __forceinline__ float dmin_a(float a, float b) { return a < b ? 1.0f : (a == b ? 0.5f : 0.0f); }
__device__ __forceinline__ float sgn(float x) { return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f); }

// The pair of pair index i, or false when the slot holds no pair (an unsolved
// problem writes -1) or an index outside its image.
__device__ __forceinline__ bool load_pair(const LossArgs& a, int64_t i, int l, int b, float4& p, float4& t,
                                          int64_t& pred_slot) {
  const int64_t q = a.query_idx[i];
  const int64_t ti = a.target_idx[i];
  const int t0 = a.tgt_offsets[b];
  const int nt = a.tgt_offsets[b + 1] - t0;
  if (q < 0 || q >= a.Q || ti < 0 || ti >= nt) return false;
  pred_slot = (static_cast<int64_t>(l) * a.B + b) * a.Q + q;
  p = __ldg(a.pred + pred_slot);
  t = __ldg(a.tgt + t0 + ti);
  return true;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  const int warp = threadIdx.x >> 5;
  if ((threadIdx.x & 31) == 0) red[warp] = v;
  __syncthreads();
  float s = 0.0f;
  if (threadIdx.x == 0) {
    for (int w = 0; w < kLossThreads / 32; ++w) s += red[w];
  }
  __syncthreads();
  return s;
}

// One CTA per (layer, image) chunk of pairs.
__global__ void __launch_bounds__(kLossThreads) box_loss_forward_kernel(const LossArgs a) {
  __shared__ float red[kLossThreads / 32];
  const int chunk = blockIdx.x;
  const int l = chunk / a.B;
  const int b = chunk - l * a.B;
  const int64_t begin = a.pair_offsets[chunk];
  const int64_t end = a.pair_offsets[chunk + 1];
  float l1 = 0.0f, lg = 0.0f;
  for (int64_t i = begin + threadIdx.x; i < end; i += kLossThreads) {
    float4 p, t;
    int64_t slot;
    if (!load_pair(a, i, l, b, p, t, slot)) continue;
    l1 += __fadd_rn(__fadd_rn(__fadd_rn(fabsf(__fsub_rn(p.x, t.x)), fabsf(__fsub_rn(p.y, t.y))),
                              fabsf(__fsub_rn(p.z, t.z))),
                    fabsf(__fsub_rn(p.w, t.w)));
    lg += __fsub_rn(1.0f, giou_terms(xyxy(p), xyxy(t)).giou);
  }
  const float s1 = block_sum(l1, red);
  const float s2 = block_sum(lg, red);
  if (threadIdx.x == 0) {
    a.l1_part[chunk] = s1;
    a.giou_part[chunk] = s2;
  }
}

__global__ void __launch_bounds__(kLossThreads) box_loss_backward_kernel(const LossArgs a) {
  const int chunk = blockIdx.x;
  const int l = chunk / a.B;
  const int b = chunk - l * a.B;
  const int64_t begin = a.pair_offsets[chunk];
  const int64_t end = a.pair_offsets[chunk + 1];
  const float g1 = a.grad_l1[l];
  const float gg = -a.grad_giou[l];  // the loss term is 1 - giou
  for (int64_t i = begin + threadIdx.x; i < end; i += kLossThreads) {
    float4 pb, tb;
    int64_t slot;
    if (!load_pair(a, i, l, b, pb, tb, slot)) continue;
    const Xyxy p = xyxy(pb), t = xyxy(tb);
    const GiouTerms g = giou_terms(p, t);
    // giou = inter / union - (hull - union) / hull = inter / union - 1 + union / hull
    const float d_uni = -g.inter / (g.uni * g.uni) + 1.0f / g.hull;
    const float d_hull = -g.uni / (g.hull * g.hull);
    const float d_inter = 1.0f / g.uni - d_uni;  // union = area_p + area_t - inter
    const float d_area = d_uni;
    // inter = clamp(iw, 0) * clamp(ih, 0), hull likewise (clamp passes the gradient at 0)
    const float diw = g.iw >= 0.0f ? d_inter * g.ihc : 0.0f;
    const float dih = g.ih >= 0.0f ? d_inter * g.iwc : 0.0f;
    const float dew = g.ew >= 0.0f ? d_hull * g.ehc : 0.0f;
    const float deh = g.eh >= 0.0f ? d_hull * g.ewc : 0.0f;
    const float pw = __fsub_rn(p.x1, p.x0), ph = __fsub_rn(p.y1, p.y0);
    // d giou / d corners of the prediction
    const float dx0 = -diw * dmax_a(p.x0, t.x0) - dew * dmin_a(p.x0, t.x0) - d_area * ph;
    const float dx1 = diw * dmin_a(p.x1, t.x1) + dew * dmax_a(p.x1, t.x1) + d_area * ph;
    const float dy0 = -dih * dmax_a(p.y0, t.y0) - deh * dmin_a(p.y0, t.y0) - d_area * pw;
    const float dy1 = dih * dmin_a(p.y1, t.y1) + deh * dmax_a(p.y1, t.y1) + d_area * pw;
    // corners -> cxcywh: x0 = cx - w/2, x1 = cx + w/2
    float4 out;
    out.x = g1 * sgn(__fsub_rn(pb.x, tb.x)) + gg * (dx0 + dx1);
    out.y = g1 * sgn(__fsub_rn(pb.y, tb.y)) + gg * (dy0 + dy1);
    out.z = g1 * sgn(__fsub_rn(pb.z, tb.z)) + gg * 0.5f * (dx1 - dx0);
    out.w = g1 * sgn(__fsub_rn(pb.w, tb.w)) + gg * 0.5f * (dy1 - dy0);
    a.grad_pred[slot] = out;
  }
}

// ---------------------------------------------------------------------------
// Classification loss over all logits with the matched classes as positives
// (SetCriterion.loss_labels, the criterion's other consumer of the indices:
// criterion.py:562 as cited at patches.py:339-341).
//
// The criterion scatters target["labels"][J] into a [B, Q] class map at the
// matched (image, query) slots and evaluates a sigmoid loss over every
// [B, Q, C] logit, positive where (q, c) is a matched query and its target's
// class.  Here one CTA covers a tile of queries of one (layer, image): it
// streams the tile's logits once, coalesced, evaluating every element as a
// negative, and corrects the matched (query, class) elements from the packed
// pairs directly (no class map, no one-hot tensor).
// Two losses, by `mode`, both summed (the caller divides by num_boxes):
//
//   FOCAL (Deformable-DETR's sigmoid_focal_loss on one-hot targets, gamma 2):
//     y = 1: alpha (1-p)^2 softplus(-x)      y = 0: (1-alpha) p^2 softplus(x)
//   IA_BCE (LW-DETR / RF-DETR IoU-aware BCE): with u = IoU(pred, target) of
//   the matched pair (box_iou: inter / union, no clamp) and
//   t = max(p^alpha u^(1-alpha), 0.01) held constant (detached):
//     y = 1: (1-t) x + softplus(-x)          y = 0: p^2 softplus(x)
//
// p = sigmoid(x), softplus(x) = max(x, 0) + log1p(exp(-|x|)).  Gradients are
// those of torch's autograd of the same expressions (t constant; the negative
// weight p^2 differentiated).  Matched labels outside [0, C) make no positive.
constexpr int kLabelThreads = 256;
constexpr int kLabelMaxTile = 4096;  // queries per CTA at most

// Queries per CTA (one partial sum each): about RFM_LABEL_LOSS_PART_ELEMS logits, a multiple of 32
// between 64 and kLabelMaxTile, so that few-class and many-class batches both give CTAs of a few
// thousand elements.
__host__ __device__ inline int label_tile_queries(int num_classes) {
  int t = RFM_LABEL_LOSS_PART_ELEMS / (num_classes > 0 ? num_classes : 1);
  t = t < 64 ? 64 : (t > kLabelMaxTile ? kLabelMaxTile : t);
  return t & ~31;
}

struct LabelArgs {
  const float* logits;          // [L, B, Q, C]
  const float4* pred;           // [L, B, Q] cxcywh (IA_BCE only)
  const int64_t* labels;        // [S]
  const float4* tgt;            // [S] cxcywh (IA_BCE only)
  const int32_t* tgt_offsets;   // [B + 1]
  const int64_t* query_idx;     // pairs
  const int64_t* target_idx;
  const int32_t* pair_offsets;  // [L * B + 1]
  int L, B, Q, C, S, tiles, tile_q;
  int mode;
  float alpha;
  float* loss_part;             // [L * B * tiles]
  int32_t* correct_part;        // [L * B * tiles] or null
  const float* grad_loss;       // [L]
  float* grad_logits;           // [L, B, Q, C]
};

// sigmoid and softplus of x from one exponent, one logarithm and one
// reciprocal: e = exp(-|x|), d = 1 + e, log1p(e) = log(d), sigmoid(x) =
// (x >= 0 ? 1 : e) / d; softplus(+-x) = max(+-x, 0) + log1p(e).
struct Sig {
  float p, q, l;  // p = sigmoid(x), q = 1 - p = sigmoid(-x), l = log1p(exp(-|x|))
};

__device__ __forceinline__ Sig sig(float x) {
  const float e = __expf(-fabsf(x));
  const float d = 1.0f + e;
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  Sig s;
  s.l = __logf(d);
  s.p = x >= 0.0f ? r : e * r;
  s.q = x >= 0.0f ? e * r : r;
  return s;
}

// IoU of two cxcywh boxes as box_iou computes it (union not clamped).
__device__ __forceinline__ float box_iou(float4 pb, float4 tb) {
  const Xyxy p = xyxy(pb), t = xyxy(tb);
  const float area_p = __fmul_rn(__fsub_rn(p.x1, p.x0), __fsub_rn(p.y1, p.y0));
  const float area_t = __fmul_rn(__fsub_rn(t.x1, t.x0), __fsub_rn(t.y1, t.y0));
  const float iw = fmaxf(__fsub_rn(fminf(p.x1, t.x1), fmaxf(p.x0, t.x0)), 0.0f);
  const float ih = fmaxf(__fsub_rn(fminf(p.y1, t.y1), fmaxf(p.y0, t.y0)), 0.0f);
  const float inter = __fmul_rn(iw, ih);
  return __fdiv_rn(inter, __fsub_rn(__fadd_rn(area_p, area_t), inter));
}

// Loss term of one logit and its derivative; `pos` marks the matched class.
__device__ __forceinline__ void label_term(const LabelArgs& a, float x, bool pos, float t, float& loss, float& grad) {
  const Sig g = sig(x);
  const float sp_pos = fmaxf(x, 0.0f) + g.l;   // softplus(x)
  const float sp_neg = fmaxf(-x, 0.0f) + g.l;  // softplus(-x)
  if (a.mode == RFM_LABEL_LOSS_FOCAL) {
    if (pos) {
      loss = a.alpha * g.q * g.q * sp_neg;
      grad = -a.alpha * g.q * g.q * (2.0f * g.p * sp_neg + g.q);
    } else {
      loss = (1.0f - a.alpha) * g.p * g.p * sp_pos;
      grad = (1.0f - a.alpha) * g.p * g.p * (2.0f * g.q * sp_pos + g.p);
    }
  } else {
    if (pos) {
      loss = (1.0f - t) * x + sp_neg;
      grad = g.p - t;
    } else {
      loss = g.p * g.p * sp_pos;
      grad = g.p * g.p * (2.0f * g.q * sp_pos + g.p);
    }
  }
}

// Matched pair k (query q) of CTA tile [q0, q0 + nq) of (layer, image) lb: its logit
// offset within the tile, its class's logit x and, for the IoU-aware loss, its
// soft target t; false when the pair is outside the tile or holds no valid
// target.  `correct` counts it when its largest logit is its class.
__device__ __forceinline__ bool load_match(const LabelArgs& a, int lb, int64_t k, int64_t q, int q0, int nq, int t0,
                                           int nt, int64_t& elem, float& x, float& t, int& correct) {
  const int64_t ti = a.target_idx[k];
  if (q < q0 || q >= q0 + nq || ti < 0 || ti >= nt) return false;
  const int64_t cls = a.labels[t0 + ti];
  if (cls < 0 || cls >= a.C) return false;
  const int64_t row_base = static_cast<int64_t>(lb) * a.Q;
  const float* row = a.logits + (row_base + q) * a.C;
  x = row[cls];
  elem = (q - q0) * a.C + cls;
  t = 0.0f;
  if (a.mode == RFM_LABEL_LOSS_IA_BCE) {
    const float p = 1.0f / (1.0f + expf(-x));
    const float u = box_iou(__ldg(a.pred + row_base + q), __ldg(a.tgt + t0 + ti));
    const float v = powf(p, a.alpha) * powf(u, 1.0f - a.alpha);
    // clamp(min=0.01) that keeps a NaN (a matched pair of two zero-area boxes has IoU 0/0), as
    // torch.clamp does: the loss is then NaN as in the unfused formula
    t = v != v ? v : fmaxf(v, 0.01f);
  }
  if (a.correct_part != nullptr) {  // top-1 (the smallest index among equal maxima)
    int best = 0;
    float bv = row[0];
    for (int c = 1; c < a.C; ++c) {
      const float v = row[c];
      if (v > bv) {
        bv = v;
        best = c;
      }
    }
    correct += best == cls ? 1 : 0;
  }
  return true;
}

// One CTA per tile of a.tile_q queries of one (layer, image).  The dense pass
// treats every logit as a negative; each matched pair then adds (forward) its
// positive term minus its negative term, or (backward) overwrites its
// gradient after the dense pass's stores.  The dense pass does not wait for the
// pairs: the two run on independent loads, and only the backward overwrite
// needs the barrier after the dense stores.
template <bool kBackward>
__global__ void __launch_bounds__(kLabelThreads) label_loss_kernel(const LabelArgs a) {
  __shared__ float red[kLabelThreads / 32];
  __shared__ int red_i[kLabelThreads / 32];
  const int tile = blockIdx.x;
  const int lb = blockIdx.y;
  const int q0 = tile * a.tile_q;
  const int nq = min(a.tile_q, a.Q - q0);
  const int b = lb % a.B;
  const int t0 = a.tgt_offsets[b];
  const int nt = a.tgt_offsets[b + 1] - t0;
  const int64_t k_begin = a.pair_offsets[lb];
  const int64_t k_end = a.pair_offsets[lb + 1];
  const int64_t base = (static_cast<int64_t>(lb) * a.Q + q0) * a.C;
  const int n = nq * a.C;
  const float g = kBackward ? a.grad_loss[lb / a.B] : 0.0f;
  // this thread's first pair is requested before the dense pass
  int64_t k = k_begin + threadIdx.x;
  int64_t q_next = k < k_end ? a.query_idx[k] : -1;
  float sum = 0.0f;
  // the dense pass is elementwise over the tile's contiguous logits: a scalar
  // head up to a 16-byte boundary, then 16-byte vectors, two in flight per
  // thread, then a scalar tail (the gradient takes the vector path when its
  // buffer has the logits' alignment)
  const float* xs = a.logits + base;
  float* gs = kBackward ? a.grad_logits + base : nullptr;
  const auto term = [&](float x, int64_t e) {
    float loss, grad;
    label_term(a, x, false, 0.0f, loss, grad);
    if (kBackward) {
      gs[e] = g * grad;
    } else {
      sum += loss;
    }
  };
  int head = static_cast<int>((4 - ((reinterpret_cast<uintptr_t>(xs) >> 2) & 3)) & 3);
  const bool vec = (reinterpret_cast<uintptr_t>(xs) & 3) == 0 &&
                   (!kBackward || ((reinterpret_cast<uintptr_t>(gs) - reinterpret_cast<uintptr_t>(xs)) & 15) == 0);
  if (!vec || head > n) head = n;
  for (int e = threadIdx.x; e < head; e += kLabelThreads) term(xs[e], e);
  const int n4 = (n - head) >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(xs + head);
  for (int i = threadIdx.x; i < n4; i += 2 * kLabelThreads) {
    const int i2 = i + kLabelThreads;
    const float4 v0 = __ldg(x4 + i);
    const float4 v1 = i2 < n4 ? __ldg(x4 + i2) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (kBackward) {
      float l, g0, g1, g2, g3;
      label_term(a, v0.x, false, 0.0f, l, g0);
      label_term(a, v0.y, false, 0.0f, l, g1);
      label_term(a, v0.z, false, 0.0f, l, g2);
      label_term(a, v0.w, false, 0.0f, l, g3);
      reinterpret_cast<float4*>(gs + head)[i] = make_float4(g * g0, g * g1, g * g2, g * g3);
      if (i2 < n4) {
        label_term(a, v1.x, false, 0.0f, l, g0);
        label_term(a, v1.y, false, 0.0f, l, g1);
        label_term(a, v1.z, false, 0.0f, l, g2);
        label_term(a, v1.w, false, 0.0f, l, g3);
        reinterpret_cast<float4*>(gs + head)[i2] = make_float4(g * g0, g * g1, g * g2, g * g3);
      }
    } else {
      term(v0.x, 0);
      term(v0.y, 0);
      term(v0.z, 0);
      term(v0.w, 0);
      if (i2 < n4) {
        term(v1.x, 0);
        term(v1.y, 0);
        term(v1.z, 0);
        term(v1.w, 0);
      }
    }
  }
  for (int e = head + 4 * n4 + threadIdx.x; e < n; e += kLabelThreads) term(xs[e], e);
  // the pairs of (l, b), strided over the threads; only the tile's are used
  int correct = 0;
  if (kBackward) __syncthreads();  // every dense store of the tile precedes the overwrites
  for (; k < k_end; k += kLabelThreads) {
    const int64_t q = q_next;
    q_next = k + kLabelThreads < k_end ? a.query_idx[k + kLabelThreads] : -1;
    int64_t elem;
    float x, t;
    if (!load_match(a, lb, k, q, q0, nq, t0, nt, elem, x, t, correct)) continue;
    float lp, gp, ln, gn;
    label_term(a, x, true, t, lp, gp);
    if (kBackward) {
      a.grad_logits[base + elem] = g * gp;
    } else {
      label_term(a, x, false, 0.0f, ln, gn);
      sum += lp - ln;
    }
  }
  if (!kBackward) {
    // fixed-order reduction: warp shuffles, then the warps' sums in order
    float v = sum;
    int c = correct;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      v += __shfl_xor_sync(kFullMask, v, o);
      c += __shfl_xor_sync(kFullMask, c, o);
    }
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
      red[warp] = v;
      red_i[warp] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.0f;
      int kk = 0;
      for (int w = 0; w < kLabelThreads / 32; ++w) {
        s += red[w];
        kk += red_i[w];
      }
      const int64_t part = static_cast<int64_t>(lb) * a.tiles + tile;
      a.loss_part[part] = s;
      if (a.correct_part != nullptr) a.correct_part[part] = kk;
    }
  }
}

int label_args(LabelArgs& a, const float* logits, const float* pred_boxes, const int64_t* labels,
               const float* tgt_boxes, const int32_t* tgt_offsets, const int64_t* query_idx,
               const int64_t* target_idx, const int32_t* pair_offsets, int L, int B, int Q, int C, int S, int mode,
               float alpha) {
  if (L < 1 || B < 1 || Q < 1 || C < 1 || S < 0 || static_cast<int64_t>(L) * B > 65535 ||
      (mode != RFM_LABEL_LOSS_FOCAL && mode != RFM_LABEL_LOSS_IA_BCE) || !(alpha >= 0.0f && alpha <= 1.0f)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (logits == nullptr || tgt_offsets == nullptr || pair_offsets == nullptr ||
      (S > 0 && labels == nullptr) ||
      (mode == RFM_LABEL_LOSS_IA_BCE && (pred_boxes == nullptr || !aligned16(pred_boxes) ||
                                         (S > 0 && (tgt_boxes == nullptr || !aligned16(tgt_boxes)))))) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  a.logits = logits;
  a.pred = reinterpret_cast<const float4*>(pred_boxes);
  a.labels = labels;
  a.tgt = reinterpret_cast<const float4*>(tgt_boxes);
  a.tgt_offsets = tgt_offsets;
  a.query_idx = query_idx;
  a.target_idx = target_idx;
  a.pair_offsets = pair_offsets;
  a.L = L;
  a.B = B;
  a.Q = Q;
  a.C = C;
  a.S = S;
  a.tile_q = label_tile_queries(C);
  a.tiles = (Q + a.tile_q - 1) / a.tile_q;
  a.mode = mode;
  a.alpha = alpha;
  a.loss_part = nullptr;
  a.correct_part = nullptr;
  a.grad_loss = nullptr;
  a.grad_logits = nullptr;
  return RFM_OK;
}

int loss_args(LossArgs& a, const float* pred_boxes, const float* tgt_boxes, const int32_t* tgt_offsets,
              const int64_t* query_idx, const int64_t* target_idx, const int32_t* pair_offsets, int L, int B,
              int Q, int S) {
  if (L < 1 || B < 1 || Q < 1 || S < 0 || static_cast<int64_t>(L) * B > 0x7fffffff) return RFM_ERR_INVALID_ARGUMENT;
  if (pred_boxes == nullptr || tgt_offsets == nullptr || pair_offsets == nullptr || !aligned16(pred_boxes) ||
      (S > 0 && (tgt_boxes == nullptr || !aligned16(tgt_boxes)))) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  a.pred = reinterpret_cast<const float4*>(pred_boxes);
  a.tgt = reinterpret_cast<const float4*>(tgt_boxes);
  a.tgt_offsets = tgt_offsets;
  a.query_idx = query_idx;
  a.target_idx = target_idx;
  a.pair_offsets = pair_offsets;
  a.L = L;
  a.B = B;
  a.Q = Q;
  a.S = S;
  a.l1_part = nullptr;
  a.giou_part = nullptr;
  a.grad_l1 = nullptr;
  a.grad_giou = nullptr;
  a.grad_pred = nullptr;
  return RFM_OK;
}

}  // namespace
}  // namespace rfm

extern "C" int rfm_box_loss_forward(const float* pred_boxes, const float* tgt_boxes, const int32_t* tgt_offsets,
                                    const int64_t* query_idx, const int64_t* target_idx,
                                    const int32_t* pair_offsets, int num_layers, int num_images, int num_queries,
                                    int sum_targets, float* l1_part, float* giou_part, void* stream) {
  using namespace rfm;
  LossArgs a;
  const int rc = loss_args(a, pred_boxes, tgt_boxes, tgt_offsets, query_idx, target_idx, pair_offsets, num_layers,
                           num_images, num_queries, sum_targets);
  if (rc != RFM_OK) return rc;
  if (l1_part == nullptr || giou_part == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  a.l1_part = l1_part;
  a.giou_part = giou_part;
  box_loss_forward_kernel<<<num_layers * num_images, kLossThreads, 0, as_stream(stream)>>>(a);
  return launch_status();
}

extern "C" int rfm_box_loss_backward(const float* pred_boxes, const float* tgt_boxes, const int32_t* tgt_offsets,
                                     const int64_t* query_idx, const int64_t* target_idx,
                                     const int32_t* pair_offsets, int num_layers, int num_images, int num_queries,
                                     int sum_targets, const float* grad_l1, const float* grad_giou,
                                     float* grad_pred, void* stream) {
  using namespace rfm;
  LossArgs a;
  const int rc = loss_args(a, pred_boxes, tgt_boxes, tgt_offsets, query_idx, target_idx, pair_offsets, num_layers,
                           num_images, num_queries, sum_targets);
  if (rc != RFM_OK) return rc;
  if (grad_l1 == nullptr || grad_giou == nullptr || grad_pred == nullptr || !aligned16(grad_pred)) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  a.grad_l1 = grad_l1;
  a.grad_giou = grad_giou;
  a.grad_pred = reinterpret_cast<float4*>(grad_pred);
  box_loss_backward_kernel<<<num_layers * num_images, kLossThreads, 0, as_stream(stream)>>>(a);
  return launch_status();
}

extern "C" int64_t rfm_label_loss_parts(int num_layers, int num_images, int num_queries, int num_classes) {
  if (num_layers < 1 || num_images < 1 || num_queries < 1 || num_classes < 1) {
    return -static_cast<int64_t>(RFM_ERR_INVALID_ARGUMENT);
  }
  const int tile = rfm::label_tile_queries(num_classes);
  return static_cast<int64_t>(num_layers) * num_images * ((num_queries + tile - 1) / tile);
}

extern "C" int rfm_label_loss_forward(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                                     const float* tgt_boxes, const int32_t* tgt_offsets, const int64_t* query_idx,
                                     const int64_t* target_idx, const int32_t* pair_offsets, int num_layers,
                                     int num_images, int num_queries, int num_classes, int sum_targets, int mode,
                                     float focal_alpha, float* loss_part, int32_t* correct_part, void* stream) {
  using namespace rfm;
  LabelArgs a;
  const int rc = label_args(a, pred_logits, pred_boxes, tgt_labels, tgt_boxes, tgt_offsets, query_idx, target_idx,
                            pair_offsets, num_layers, num_images, num_queries, num_classes, sum_targets, mode,
                            focal_alpha);
  if (rc != RFM_OK) return rc;
  if (loss_part == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  a.loss_part = loss_part;
  a.correct_part = correct_part;
  const dim3 grid(static_cast<unsigned>(a.tiles), static_cast<unsigned>(num_layers * num_images));
  label_loss_kernel<false><<<grid, kLabelThreads, 0, as_stream(stream)>>>(a);
  return launch_status();
}

extern "C" int rfm_label_loss_backward(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                                      const float* tgt_boxes, const int32_t* tgt_offsets, const int64_t* query_idx,
                                      const int64_t* target_idx, const int32_t* pair_offsets, int num_layers,
                                      int num_images, int num_queries, int num_classes, int sum_targets, int mode,
                                      float focal_alpha, const float* grad_loss, float* grad_logits, void* stream) {
  using namespace rfm;
  LabelArgs a;
  const int rc = label_args(a, pred_logits, pred_boxes, tgt_labels, tgt_boxes, tgt_offsets, query_idx, target_idx,
                            pair_offsets, num_layers, num_images, num_queries, num_classes, sum_targets, mode,
                            focal_alpha);
  if (rc != RFM_OK) return rc;
  if (grad_loss == nullptr || grad_logits == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  a.grad_loss = grad_loss;
  a.grad_logits = grad_logits;
  const dim3 grid(static_cast<unsigned>(a.tiles), static_cast<unsigned>(num_layers * num_images));
  label_loss_kernel<true><<<grid, kLabelThreads, 0, as_stream(stream)>>>(a);
  return launch_status();
}
