// Fused matcher cost kernel: focal class cost + L1 + GIoU, one pass, HBM-bound.
//
// Replaces the Triton kernel _matcher_cost_kernel (kernels_matcher.py:56-176)
// and the padded->compact torch.cat of the triton_matcher patch
// (patches.py:137-149): the compact [Q, sum T] matrix of every decoder layer is
// written directly, so there is no padded intermediate and no copy.
//
// Two output layouts.  TARGET-MAJOR (the transpose, out[l][col][q]) is the one
// the fused matcher step uses: one CTA covers 64 consecutive target rows (8 when
// 64-row CTAs would not fill the GPU twice, as in the production step; runs
// of one image each) and a 256-query tile; each thread owns two consecutive
// queries (one 8-byte vector of every output row), loads their boxes and logits
// once per image run (the next run's while computing the current one),
// evaluates the focal cost once per class when there are at most four classes,
// and then walks the run's targets (staged in shared memory, read as
// broadcasts), so every warp store is a coalesced 256-byte write along the row
// and every input is read once per run.  Two queries per thread keep the kernel
// near 72 registers, several CTAs per SM, which hides more latency than wider
// per-thread tiles do.
//
// QUERY-MAJOR (the compact matrix itself, out[l][q][col]) serves the drop-in
// cost-matrix call.  The same kernel computes the same tiles (32 target rows x
// 256 queries) into shared memory instead, query-major, and then writes each
// query row's 32 columns out as one coalesced store; any ld >= S is accepted
// and the pad columns are written with 0.
//
// Arithmetic.  Every operation is explicitly rounded: scalar add/sub/mul.rn,
// packed f32x2 ops (same per-lane rounding) and explicit FMAs.  ptxas contracts
// a packed multiply feeding a packed add into an FMA even with .rn, so every
// product that is added to something is written as an explicit FMA, in both
// layouts: union = fma(-iw, ih, area_p + area_t), hull - union, the GIoU
// difference and the weighted sum.  The L1 term follows the reference chain
// (kernels_matcher.py:98-120) bit for bit, and so do the boxes' areas.  The
// intersection and hull extents come from the same centre and half-width
// differences as L1, by the interval identities min(a1,b1) - max(a0,b0) =
// ha + hb - max(|ca - cb|, |ha - hb|) and max(a1,b1) - min(a0,b0) = ha + hb +
// max(|ca - cb|, |ha - hb|) (centres c, half-widths h): the reference's corner
// min/max, rounded differently (within an ulp of the coordinates).  Quotients
// are a * rcp(b); the focal term uses fast exp/log.  All of it is well inside
// the 1e-5 relative bar, and both layouts come out of the same code, so they
// hold bit-identical matrices.
#include "rfm_common.cuh"

namespace rfm {
namespace {

constexpr float kBoxEps = 1e-7f;  // kernels_matcher.py:53

struct CostArgs {
  const float* logits;   // [L, B, Q, C]
  const float4* pboxes;  // [L, B, Q] cxcywh
  const int64_t* labels; // [S]
  const float4* tboxes;  // [S] cxcywh
  const int32_t* offsets;  // [B + 1]
  int B, Q, C, S;
  int64_t ld;
  float w_class, w_bbox, w_giou, alpha, alpha_m1;
  float* out;            // [L, Q, ld]
  int* reset_word;       // target-major only: set to 0 by one thread (a solver counter), or null
};

struct Corners {
  float x0, y0, x1, y1, area;
};

// cxcywh -> xyxy and area computed from the corners, as
// box_cxcywh_to_xyxy + box_area do (kernels_matcher.py:106-116).
__device__ __forceinline__ Corners corners(const float4 b) {
  Corners c;
  const float hw = __fmul_rn(0.5f, b.z);
  const float hh = __fmul_rn(0.5f, b.w);
  c.x0 = __fsub_rn(b.x, hw);
  c.y0 = __fsub_rn(b.y, hh);
  c.x1 = __fadd_rn(b.x, hw);
  c.y1 = __fadd_rn(b.y, hh);
  c.area = __fmul_rn(__fsub_rn(c.x1, c.x0), __fsub_rn(c.y1, c.y0));
  return c;
}

// 1 / b by PTX rcp.approx (max error about 1 ulp); quotients are a * rcp(b) with
// one rounded multiply.  b is never below the 1e-7 clamp, so flushing
// subnormals is moot.
__device__ __forceinline__ float rcp_approx(float b) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(b));
  return r;
}


// alpha (1-p)^2 (-logsigmoid(x)) - (1-alpha) p^2 (-logsigmoid(-x)), p = sigmoid(x)
// (kernels_matcher.py:257-260), with logsigmoid(x) = min(x, 0) - log1p(exp(-|x|)).
// Fast exponent and logarithm: e = exp(-|x|), log1p(e) = log(1 + e),
// sigmoid(x) = s * rcp(1 + e) with s = (x >= 0 ? 1 : e), 1 - p = fma(-s, rcp, 1),
// and the final difference as fma(alpha (1-p)^2, -logsigmoid(x), (alpha-1) p^2
// (-logsigmoid(-x))); within ~1e-6 of the exact chain.  Every rounding step is
// explicit, and focal_cost2 evaluates the same operations on two logits at once,
// so every call site produces identical bits.  alpha_m1 = -(1 - alpha).
__device__ __forceinline__ float focal_cost(float x, float alpha, float alpha_m1) {
  const float e = __expf(-fabsf(x));
  const float onep = __fadd_rn(1.0f, e);
  const float l = __logf(onep);
  const float s = x >= 0.0f ? 1.0f : e;
  const float r = rcp_approx(onep);
  const float p = __fmul_rn(s, r);
  const float q = __fmaf_rn(-s, r, 1.0f);
  const float mpos = __fsub_rn(l, fminf(x, 0.0f));
  const float mneg = __fsub_rn(l, fminf(-x, 0.0f));
  const float nneg = __fmul_rn(__fmul_rn(alpha_m1, __fmul_rn(p, p)), mneg);
  return __fmaf_rn(__fmul_rn(alpha, __fmul_rn(q, q)), mpos, nneg);
}

// Largest image b in [lo, hi) with offsets[b] <= col, given offsets[lo] <= col
// < offsets[hi] (images with no targets are skipped).
__device__ __forceinline__ int image_in_range(const int32_t* offsets, int lo, int hi, int col) {
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(offsets + mid) <= col) {
      lo = mid;
    } else {
      hi = mid;
    }
  }
  return lo;
}

// Image lookup for a CTA whose targets start at `first`.  The CTA narrows the
// image of `first` with a 128-way search (no round at all for B <= 128: each
// round is one load per thread, against the ten dependent loads of a binary
// search over 1024 images), then stages offsets[lo .. lo + kImageWindow] in
// shared memory; image_in_window() answers from there.  Needs >= 128 threads,
// called by all of them.
constexpr int kImageWindow = 128;

__device__ __forceinline__ int stage_image_window(const int32_t* offsets, int B, int first, int* s_off,
                                                  int tid, int nthreads) {
  int lo = 0, hi = B;  // offsets[lo] <= first < offsets[hi] = S
  while (hi - lo > kImageWindow) {
    const int stride = (hi - lo + kImageWindow - 1) / kImageWindow;
    const int idx = lo + tid * stride;
    const int below = tid < kImageWindow && idx < hi && __ldg(offsets + idx) <= first;
    const int count = __syncthreads_count(below);  // a prefix of the probes: offsets are sorted
    lo += (count - 1) * stride;
    hi = min(hi, lo + stride);
  }
  for (int e = tid; e <= kImageWindow; e += nthreads) s_off[e] = __ldg(offsets + min(lo + e, B));
  __syncthreads();
  return lo;
}

// Image of target `col` >= first; past the window (more than kImageWindow
// images, most of them empty, before col) it searches global memory.
__device__ __forceinline__ int image_in_window(const int* s_off, int lo, const int32_t* offsets, int B,
                                               int col) {
  if (lo + kImageWindow < B && col >= s_off[kImageWindow]) {
    return image_in_range(offsets, lo + kImageWindow, B, col);
  }
  int l = 0, h = min(kImageWindow, B - lo);  // s_off[l] <= col < s_off[h]
  while (h - l > 1) {
    const int mid = (l + h) >> 1;
    if (s_off[mid] <= col) {
      l = mid;
    } else {
      h = mid;
    }
  }
  return lo + l;
}

constexpr int kTmThreads = 128;  // 2 queries each: 256 queries per CTA
constexpr int kQpt = 2;          // queries per thread (one f32x2 pair)
constexpr int kTmCols = 64;      // target rows per CTA (may span several images)
constexpr int kTmColsSmall = 8;  // ... for batches too small to fill the GPU twice with 64-row CTAs
constexpr int kQmCols = 32;      // target rows per CTA in the query-major layout (its tile is in shared memory)
constexpr int kSmallClasses = 4;

// Packed float32 pairs: two queries per instruction (sm_100 f32x2 pipe), each
// half rounded exactly as the scalar instruction would round it.
__device__ __forceinline__ unsigned long long pk(float2 a) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
__device__ __forceinline__ float2 upk(unsigned long long r) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
  return a;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
  return upk(r);
}
__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
  return upk(r);
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)));
  return upk(r);
}
__device__ __forceinline__ float2 dup2(float x) { return make_float2(x, x); }

// Shared per-target data of the inner loop (32 bytes, two broadcast loads).
struct TargetRow {
  float4 box;  // cx, cy, w / 2, h / 2
  float area;  // of the xyxy corners, as box_area computes it
  int label;
  int image;
  int plain;   // w >= 0, h >= 0 and area >= 2e-7: the clamps are no-ops
};

// Prediction data of one pair of queries of one image: centres, half extents
// and the corners' area.
struct PredPair {
  float2 cx, cy, hw, hh, area;
};

__device__ __forceinline__ PredPair pred_pair(const float4 a, const float4 b) {
  PredPair p;
  p.cx = make_float2(a.x, b.x);
  p.cy = make_float2(a.y, b.y);
  p.hw = mul2(dup2(0.5f), make_float2(a.z, b.z));
  p.hh = mul2(dup2(0.5f), make_float2(a.w, b.w));
  const float2 pw = sub2(add2(p.cx, p.hw), sub2(p.cx, p.hw));
  const float2 ph = sub2(add2(p.cy, p.hh), sub2(p.cy, p.hh));
  p.area = mul2(pw, ph);
  return p;
}

__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  unsigned long long r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(pk(a)), "l"(pk(b)), "l"(pk(c)));
  return upk(r);
}

// focal_cost of two logits: the same operations, packed where they are add, sub,
// mul or fma (no packed product feeds a packed add, so nothing is contracted).
__device__ __forceinline__ float2 focal_cost2(float2 x, float alpha, float alpha_m1) {
  const float2 e = make_float2(__expf(-fabsf(x.x)), __expf(-fabsf(x.y)));
  const float2 onep = add2(dup2(1.0f), e);
  const float2 l = make_float2(__logf(onep.x), __logf(onep.y));
  const float2 sv = make_float2(x.x >= 0.0f ? 1.0f : e.x, x.y >= 0.0f ? 1.0f : e.y);
  const float2 r = make_float2(rcp_approx(onep.x), rcp_approx(onep.y));
  const float2 p = mul2(sv, r);
  const float2 q = fma2(make_float2(-sv.x, -sv.y), r, dup2(1.0f));
  const float2 mpos = sub2(l, make_float2(fminf(x.x, 0.0f), fminf(x.y, 0.0f)));
  const float2 mneg = sub2(l, make_float2(fminf(-x.x, 0.0f), fminf(-x.y, 0.0f)));
  const float2 nneg = mul2(mul2(dup2(alpha_m1), mul2(p, p)), mneg);
  return fma2(mul2(dup2(alpha), mul2(q, q)), mpos, nneg);
}

// Cost of one target against a pair of queries (two packed lanes).  With
// kUnclamped the hull and 1e-7 clamps are skipped: the caller guarantees they
// are no-ops (both boxes have non-negative width and height, so the hull
// extents are >= 0, and the target's area is >= 2e-7, so union and hull exceed
// 1e-7), which leaves every result bit-identical to the clamped formula.
template <bool kUnclamped>
__device__ __forceinline__ float2 pair_cost2(const PredPair& p, const TargetRow& t, float2 wcls,
                                             const CostArgs& a) {
  const float2 dcx = sub2(p.cx, dup2(t.box.x));
  const float2 dcy = sub2(p.cy, dup2(t.box.y));
  const float2 dhx = sub2(p.hw, dup2(t.box.z));
  const float2 dhy = sub2(p.hh, dup2(t.box.w));
  // L1 over cxcywh in the reference's order ((|dcx| + |dcy|) + |dw|) + |dh|;
  // |dw| = 2 |dw / 2| exactly (halving and doubling are exact for normal floats)
  const float2 l1 = make_float2(
      __fmaf_rn(2.0f, fabsf(dhy.x), __fmaf_rn(2.0f, fabsf(dhx.x), __fadd_rn(fabsf(dcx.x), fabsf(dcy.x)))),
      __fmaf_rn(2.0f, fabsf(dhy.y), __fmaf_rn(2.0f, fabsf(dhx.y), __fadd_rn(fabsf(dcx.y), fabsf(dcy.y)))));
  // Two intervals of half-widths a and b whose centres are d apart overlap by
  // a + b - max(|d|, |a - b|) and span a + b + max(|d|, |a - b|) (the min/max
  // of their corners, rewritten): both extents come from the L1 differences.
  const float2 mx = make_float2(fmaxf(fabsf(dcx.x), fabsf(dhx.x)), fmaxf(fabsf(dcx.y), fabsf(dhx.y)));
  const float2 my = make_float2(fmaxf(fabsf(dcy.x), fabsf(dhy.x)), fmaxf(fabsf(dcy.y), fabsf(dhy.y)));
  const float2 sx = add2(p.hw, dup2(t.box.z));
  const float2 sy = add2(p.hh, dup2(t.box.w));
  const float2 iw = sub2(sx, mx);
  const float2 ih = sub2(sy, my);
  const float2 iwc = make_float2(fmaxf(iw.x, 0.f), fmaxf(iw.y, 0.f));
  const float2 ihc = make_float2(fmaxf(ih.x, 0.f), fmaxf(ih.y, 0.f));
  const float2 inter = mul2(iwc, ihc);
  const float2 uni = fma2(make_float2(-iwc.x, -iwc.y), ihc, add2(p.area, dup2(t.area)));
  const float2 ew = add2(sx, mx);  // hull extents
  const float2 eh = add2(sy, my);
  float2 ewc = ew, ehc = eh, uc = uni;
  if (!kUnclamped) {
    ewc = make_float2(fmaxf(ew.x, 0.f), fmaxf(ew.y, 0.f));
    ehc = make_float2(fmaxf(eh.x, 0.f), fmaxf(eh.y, 0.f));
    uc = make_float2(fmaxf(uni.x, kBoxEps), fmaxf(uni.y, kBoxEps));
  }
  const float2 hull = mul2(ewc, ehc);
  const float2 gap = fma2(ewc, ehc, make_float2(-uni.x, -uni.y));
  float2 hc = hull;
  if (!kUnclamped) hc = make_float2(fmaxf(hull.x, kBoxEps), fmaxf(hull.y, kBoxEps));
  const float2 iou = mul2(inter, make_float2(rcp_approx(uc.x), rcp_approx(uc.y)));
  const float2 giou = fma2(make_float2(-gap.x, -gap.y), make_float2(rcp_approx(hc.x), rcp_approx(hc.y)), iou);
  return fma2(dup2(-a.w_giou), giou, fma2(dup2(a.w_bbox), l1, wcls));
}

// Loads of the next image's predictions, issued before they are needed.
template <int NCLS>
struct PredRaw {
  float4 box[kQpt];
  float lg[kQpt][NCLS > 0 ? NCLS : 1];
};

template <int NCLS>
__device__ __forceinline__ void load_raw(PredRaw<NCLS>& r, const CostArgs& a, int64_t pbase, int q0) {
#pragma unroll
  for (int k = 0; k < kQpt; ++k) {
    const int q = q0 + k < a.Q ? q0 + k : a.Q - 1;  // pad queries reuse a valid row
    r.box[k] = __ldg(a.pboxes + pbase + q);
    if (NCLS > 0) {
#pragma unroll
      for (int c = 0; c < NCLS; ++c) r.lg[k][c] = __ldg(a.logits + (pbase + q) * NCLS + c);
    }
  }
}

__device__ __forceinline__ void st_shared(unsigned addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Costs of targets [c_begin, c_end) of one image run against the thread's two
// queries: one 8-byte store per target row of the target-major matrix, or
// (kQM) two 4-byte stores into the CTA's query-major shared-memory tile, whose
// thread rows start at the shared-memory byte address `tile` (32-bit shared
// addressing: the tile's stores need no 64-bit address arithmetic).
template <int NCLS, bool kUnclamped, bool kTail, bool kQM>
__device__ __forceinline__ void cost_targets(const TargetRow* s_t, int c_begin, int c_end, float* out_row,
                                             const PredPair& p01, const float2 (&wcls01)[kSmallClasses],
                                             int q0, int64_t pbase, const CostArgs& a, unsigned tile, int pitch) {
  float* dst = kQM ? nullptr : out_row + static_cast<int64_t>(c_begin) * a.ld;
  const int64_t step = kQM ? 0 : a.ld;
  unsigned sdst = tile + 4u * static_cast<unsigned>(c_begin);
#pragma unroll 2
  for (int c = c_begin; c < c_end; ++c, dst += step, sdst += 4u) {
    const TargetRow t = s_t[c];
    float2 w01;
    if (NCLS > 0) {
      w01 = wcls01[0];
#pragma unroll
      for (int cl = 1; cl < NCLS; ++cl) w01 = t.label == cl ? wcls01[cl] : w01;
    } else {
      float f[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int q = q0 + k < a.Q ? q0 + k : a.Q - 1;
        f[k] = __fmul_rn(a.w_class, focal_cost(__ldg(a.logits + (pbase + q) * a.C + t.label), a.alpha,
                                               a.alpha_m1));
      }
      w01 = make_float2(f[0], f[1]);
    }
    float2 r01 = pair_cost2<kUnclamped>(p01, t, w01, a);
    if (kQM) {  // rows of queries q0 and q0 + 1 of the tile (a query past Q is never written out)
      st_shared(sdst, r01.x);
      st_shared(sdst + 4u * static_cast<unsigned>(pitch), r01.y);
    } else {
      if (kTail && q0 + 2 > a.Q) {  // zero the pad queries (q >= Q, up to ld) of the last tile
        if (q0 >= a.Q) r01.x = 0.f;
        r01.y = 0.f;
      }
      *reinterpret_cast<float2*>(dst) = r01;
    }
  }
}

// One CTA: kCols consecutive target rows x 256 queries.  Target-major: every
// cost goes straight to its row.  Query-major (kQM, the compact [Q, ld] matrix):
// the tile is built in shared memory, query-major with a pitch of kCols + 1
// floats, then each query row's kCols costs leave as one coalesced store of
// consecutive columns; a CTA past the last target only zeroes its pad columns.
// The arithmetic is the same in both, so the two layouts hold identical bits.
template <int NCLS, int kCols, bool kQM>
__global__ void __launch_bounds__(kTmThreads) cost_tmajor_kernel(const CostArgs a) {
  // A solver launched after this kernel with programmatic stream serialization
  // may start its prologue now; it waits for this grid's completion (and its
  // stores) before it reads the matrix.
  asm volatile("griddepcontrol.launch_dependents;");
  if (!kQM && a.reset_word != nullptr && (blockIdx.x | blockIdx.y | blockIdx.z | threadIdx.x) == 0) {
    *a.reset_word = 0;
  }
  constexpr int kPitch = kCols + 1;
  __shared__ float s_tile[kQM ? kQpt * kTmThreads * kPitch : 1];
  if (kQM && static_cast<int64_t>(blockIdx.x) * kCols >= a.S) {
    // pad columns only: zero [c_begin, min(c_begin + kCols, ld)) of every query row of the tile
    const int64_t c0 = static_cast<int64_t>(blockIdx.x) * kCols;
    const int width = static_cast<int>(min(static_cast<int64_t>(kCols), a.ld - c0));
    const int qt0 = blockIdx.y * kTmThreads * kQpt;
    for (int e = threadIdx.x; e < kTmThreads * kQpt * kCols; e += kTmThreads) {
      const int ql = e / kCols, c = e - ql * kCols;
      if (c < width && qt0 + ql < a.Q) {
        a.out[(static_cast<int64_t>(blockIdx.z) * a.Q + qt0 + ql) * a.ld + c0 + c] = 0.0f;
      }
    }
    return;
  }
  __shared__ TargetRow s_t[kCols];
  __shared__ int s_seg[kCols + 1];
  __shared__ int s_nseg;
  __shared__ int s_all_plain;
  __shared__ int s_off[kImageWindow + 1];
  const int layer = blockIdx.z;
  const int c_begin = blockIdx.x * kCols;
  const int n = min(kCols, a.S - c_begin);
  const int tid = threadIdx.x;
  static_assert(kCols <= kTmThreads, "one staged target per thread");
  // this thread's target is requested first; its latency overlaps the image search
  const bool has_target = tid < n;
  float4 tbox = make_float4(0.f, 0.f, 0.f, 0.f);
  int64_t tlabel = 0;
  if (has_target) {
    tbox = __ldg(a.tboxes + c_begin + tid);
    tlabel = __ldg(a.labels + c_begin + tid);
  }
  const int win_lo = stage_image_window(a.offsets, a.B, c_begin, s_off, tid, kTmThreads);
  const int q0 = (blockIdx.y * kTmThreads + tid) * kQpt;
  const int64_t layer_base = static_cast<int64_t>(layer) * a.B;
  // the first run's predictions are requested before the targets are staged
  PredRaw<NCLS> raw;
  load_raw<NCLS>(raw, a, (layer_base + image_in_window(s_off, win_lo, a.offsets, a.B, c_begin)) * a.Q, q0);

  // stage this CTA's targets ...
  if (has_target) {
    const int col = c_begin + tid;
    TargetRow t;
    const Corners cn = corners(tbox);
    t.box = make_float4(tbox.x, tbox.y, __fmul_rn(0.5f, tbox.z), __fmul_rn(0.5f, tbox.w));
    t.area = cn.area;
    t.label = static_cast<int>(tlabel < 0 ? 0 : (tlabel >= a.C ? a.C - 1 : tlabel));
    t.image = image_in_window(s_off, win_lo, a.offsets, a.B, col);
    t.plain = (tbox.z >= 0.0f && tbox.w >= 0.0f && cn.area >= 2e-7f) ? 1 : 0;
    s_t[tid] = t;
  }
  __syncthreads();
  // ... and split them into runs of one image (warp 0)
  if (tid < 32) {
    int count = 0;
    bool every = true;
    for (int base0 = 0; base0 < n; base0 += 32) {
      const int c = base0 + tid;
      const bool in = c < n;
      const bool start = in && (c == 0 || s_t[c].image != s_t[c - 1].image);
      const unsigned starts = __ballot_sync(kFullMask, start);
      if (start) s_seg[count + __popc(starts & ((1u << tid) - 1u))] = c;
      count += __popc(starts);
      every = __all_sync(kFullMask, !in || s_t[c].plain) && every;
    }
    if (tid == 0) {
      s_nseg = count;
      s_seg[count] = n;
      s_all_plain = every ? 1 : 0;
    }
  }
  __syncthreads();
  if (!kQM && q0 >= a.ld) return;
  const int nseg = (kQM && q0 >= a.Q) ? 0 : s_nseg;  // query-major: queries past Q are not computed
  const bool all_plain = s_all_plain != 0;
  float* out_row = kQM ? nullptr : a.out + (static_cast<int64_t>(layer) * a.S + c_begin) * a.ld + q0;
  const unsigned tile_row =
      static_cast<unsigned>(__cvta_generic_to_shared(s_tile)) + (kQM ? 4u * tid * kQpt * kPitch : 0u);
  for (int sg = 0; sg < nseg; ++sg) {
    const int img = s_t[s_seg[sg]].image;
    const int64_t pbase = (layer_base + img) * a.Q;
    const PredPair p01 = pred_pair(raw.box[0], raw.box[1]);
    bool preds_plain = true;
#pragma unroll
    for (int k = 0; k < 2; ++k) preds_plain = preds_plain && raw.box[k].z >= 0.0f && raw.box[k].w >= 0.0f;
    float2 wcls01[kSmallClasses];
    if (NCLS > 0) {
#pragma unroll
      for (int c = 0; c < NCLS; ++c) {
        wcls01[c] = mul2(dup2(a.w_class), focal_cost2(make_float2(raw.lg[0][c], raw.lg[1][c]), a.alpha, a.alpha_m1));
      }
    }
    if (sg + 1 < nseg) {
      load_raw<NCLS>(raw, a, (layer_base + s_t[s_seg[sg + 1]].image) * a.Q, q0);
    }
    // one uniform choice per image run: clamp-free when every box of the run is
    // plain, pad-query zeroing only in the last query tile
    if (preds_plain && all_plain && q0 + 2 <= a.Q) {
      cost_targets<NCLS, true, false, kQM>(s_t, s_seg[sg], s_seg[sg + 1], out_row, p01, wcls01, q0, pbase, a,
                                          tile_row, kPitch);
    } else {
      cost_targets<NCLS, false, true, kQM>(s_t, s_seg[sg], s_seg[sg + 1], out_row, p01, wcls01, q0, pbase, a,
                                          tile_row, kPitch);
    }
  }
  if (kQM) {
    // the tile out, query-major: warp w writes query rows w, w + 4, ...; lane c
    // column c_begin + c (the row's real columns, then its pad columns with 0)
    __syncthreads();
    static_assert(!kQM || kCols <= 32, "one column per lane");
    const int width = static_cast<int>(min(static_cast<int64_t>(kCols), a.ld - c_begin));
    const int qt0 = blockIdx.y * kTmThreads * kQpt;
    const int lane = tid & 31, warp = tid >> 5;
    const int rows = min(kTmThreads * kQpt, a.Q - qt0);
    constexpr int kWarps = kTmThreads / 32;
    if (lane < width) {
      float* dst = a.out + (static_cast<int64_t>(layer) * a.Q + qt0 + warp) * a.ld + c_begin + lane;
      const int64_t row_step = kWarps * a.ld;
      const float* src = s_tile + warp * kPitch + lane;
      for (int ql = warp; ql < rows; ql += kWarps, dst += row_step, src += kWarps * kPitch) {
        *dst = lane < n ? *src : 0.0f;
      }
    }
  }
}

template <int kCols, bool kQM>
void launch_tmajor(const CostArgs& a, dim3 grid, int num_classes, cudaStream_t stream) {
  switch (num_classes) {
    case 1: cost_tmajor_kernel<1, kCols, kQM><<<grid, kTmThreads, 0, stream>>>(a); break;
    case 2: cost_tmajor_kernel<2, kCols, kQM><<<grid, kTmThreads, 0, stream>>>(a); break;
    case 3: cost_tmajor_kernel<3, kCols, kQM><<<grid, kTmThreads, 0, stream>>>(a); break;
    case 4: cost_tmajor_kernel<4, kCols, kQM><<<grid, kTmThreads, 0, stream>>>(a); break;
    default: cost_tmajor_kernel<0, kCols, kQM><<<grid, kTmThreads, 0, stream>>>(a); break;
  }
}

}  // namespace
}  // namespace rfm

namespace rfm {
int cost_run(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
             const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
             int num_queries, int num_classes, int sum_targets, int64_t ld, int layout,
             float cost_class, float cost_bbox, float cost_giou, float focal_alpha, float* out,
             int* reset_word, void* stream) {
  if (num_layers < 1 || num_layers > 65535 || num_images < 1 || num_queries < 1 ||
      num_classes < 1 || sum_targets < 0) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (layout == RFM_LAYOUT_QUERY_MAJOR) {
    if (ld < sum_targets) return RFM_ERR_INVALID_ARGUMENT;
    if (ld == 0) return RFM_OK;
  } else if (layout == RFM_LAYOUT_TARGET_MAJOR) {
    if (ld < num_queries || (ld & 3) != 0) return RFM_ERR_INVALID_ARGUMENT;
    if (sum_targets == 0) return RFM_OK;
    if (out != nullptr && !aligned16(out)) return RFM_ERR_INVALID_ARGUMENT;
  } else {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (out == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  if (sum_targets > 0 &&
      (pred_logits == nullptr || pred_boxes == nullptr || tgt_labels == nullptr ||
       tgt_boxes == nullptr || tgt_offsets == nullptr || !aligned16(pred_boxes) ||
       !aligned16(tgt_boxes))) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(num_images) * num_queries * num_classes > (int64_t(1) << 40)) {
    return RFM_ERR_UNSUPPORTED;
  }

  CostArgs a;
  a.logits = pred_logits;
  a.pboxes = reinterpret_cast<const float4*>(pred_boxes);
  a.labels = tgt_labels;
  a.tboxes = reinterpret_cast<const float4*>(tgt_boxes);
  a.offsets = tgt_offsets;
  a.B = num_images;
  a.Q = num_queries;
  a.C = num_classes;
  a.S = sum_targets;
  a.ld = ld;
  a.w_class = cost_class;
  a.w_bbox = cost_bbox;
  a.w_giou = cost_giou;
  a.alpha = focal_alpha;
  // torch multiplies by the Python scalar (1 - alpha), rounded once to float32
  a.alpha_m1 = -static_cast<float>(1.0 - static_cast<double>(focal_alpha));
  a.out = out;
  a.reset_word = reset_word;

  if (layout == RFM_LAYOUT_TARGET_MAJOR) {
    const int64_t gy = (ld / kQpt + kTmThreads - 1) / kTmThreads;
    // 64 target rows per CTA, or 8 when that leaves fewer than two CTAs per SM
    // (the production step: a few hundred CTAs, each then a quarter as long)
    const int64_t gx_big = (static_cast<int64_t>(sum_targets) + kTmCols - 1) / kTmCols;
    const bool small = gx_big * gy * num_layers < 2 * static_cast<int64_t>(device_sm_count());
    const int cols = small ? kTmColsSmall : kTmCols;
    const int64_t gx = (static_cast<int64_t>(sum_targets) + cols - 1) / cols;
    if (gy > 65535 || gx > 0x7fffffff) return RFM_ERR_UNSUPPORTED;
    const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy),
                    static_cast<unsigned>(num_layers));
    if (small) {
      launch_tmajor<kTmColsSmall, false>(a, grid, num_classes, as_stream(stream));
    } else {
      launch_tmajor<kTmCols, false>(a, grid, num_classes, as_stream(stream));
    }
    return launch_status();
  }

  // query-major: the same tiles (32 target rows, or 8 for small batches) computed
  // into shared memory and written out transposed; the grid covers every column
  // up to ld so the pad columns are zeroed
  const int64_t gy = (static_cast<int64_t>(num_queries) + kQpt * kTmThreads - 1) / (kQpt * kTmThreads);
  const int64_t gx_big = (static_cast<int64_t>(sum_targets) + kQmCols - 1) / kQmCols;
  const bool small = gx_big * gy * num_layers < 2 * static_cast<int64_t>(device_sm_count());
  const int cols = small ? kTmColsSmall : kQmCols;
  const int64_t gx = (ld + cols - 1) / cols;
  if (gy > 65535 || gx > 0x7fffffff) return RFM_ERR_UNSUPPORTED;
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), static_cast<unsigned>(num_layers));
  if (small) {
    launch_tmajor<kTmColsSmall, true>(a, grid, num_classes, as_stream(stream));
  } else {
    launch_tmajor<kQmCols, true>(a, grid, num_classes, as_stream(stream));
  }
  return launch_status();
}

}  // namespace rfm

extern "C" int rfm_cost(const float* pred_logits, const float* pred_boxes,
                        const int64_t* tgt_labels, const float* tgt_boxes,
                        const int32_t* tgt_offsets, int num_layers, int num_images,
                        int num_queries, int num_classes, int sum_targets, int64_t ld, int layout,
                        float cost_class, float cost_bbox, float cost_giou, float focal_alpha,
                        float* out, void* stream) {
  return rfm::cost_run(pred_logits, pred_boxes, tgt_labels, tgt_boxes, tgt_offsets, num_layers, num_images,
                       num_queries, num_classes, sum_targets, ld, layout, cost_class, cost_bbox, cost_giou,
                       focal_alpha, out, nullptr, stream);
}
