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
