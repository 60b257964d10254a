// Fused matcher cost kernel: focal class cost + L1 + GIoU, one pass, HBM-bound.
//
// Replaces the Triton kernel _matcher_cost_kernel (kernels_matcher.py:56-176)
// and the padded->compact torch.cat of the triton_matcher patch
// (patches.py:137-149): the compact [Q, sum T] matrix of every decoder layer is
// written directly, so there is no padded intermediate and no copy.
//
// Work mapping.  Each thread owns four consecutive columns of the output (one
// 16-byte vector) and walks a strip of rows.  The target data of its columns
// (box, xyxy corners, area, clamped label, owning image) is loaded once into
// registers and reused for every row; the per-(image, query) prediction data
// (box and the logit at the target's class) comes through L1, where the
// neighbouring columns of the same image hit it again.  Stores are 128-bit,
// coalesced along the row when the row stride ld is a multiple of 4 (every
// row then starts 16-byte aligned; the caller pads ld and the pad columns are
// written with 0); any other ld takes a scalar-store variant.
//
// Arithmetic.  The box terms use explicitly rounded float32 intrinsics in the
// reference chain's order of operations (no FMA contraction), so they are
// bit-identical to a float32 evaluation of kernels_matcher.py:98-127 and :264;
// the focal term uses CUDA's expf/log1pf.
#include "rfm_common.cuh"

namespace rfm {
namespace {

constexpr int kThreads = 256;
constexpr int kRowsPerThread = 8;
constexpr float kBoxEps = 1e-7f;  // kernels_matcher.py:53

struct CostArgs {
  const float* logits;   // [L, B, Q, C]
  const float4* pboxes;  // [L, B, Q] cxcywh
  const int64_t* labels; // [S]
  const float4* tboxes;  // [S] cxcywh
  const int32_t* offsets;  // [B + 1]
  int B, Q, C, S;
  int64_t ld;
  int rows_per_cta;
  float w_class, w_bbox, w_giou, alpha, one_minus_alpha;
  float* out;            // [L, Q, ld]
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

// alpha (1-p)^2 (-logsigmoid(x)) - (1-alpha) p^2 (-logsigmoid(-x)), p = sigmoid(x)
// (kernels_matcher.py:257-260; logsigmoid(x) = min(x, 0) - log1p(exp(-|x|))).
__device__ __forceinline__ float focal_cost(float x, float alpha, float one_minus_alpha) {
  const float p = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
  const float l = log1pf(expf(-fabsf(x)));
  const float ls_pos = __fsub_rn(fminf(x, 0.0f), l);
  const float ls_neg = __fsub_rn(fminf(-x, 0.0f), l);
  const float q = __fsub_rn(1.0f, p);
  const float neg = __fmul_rn(__fmul_rn(one_minus_alpha, __fmul_rn(p, p)), -ls_neg);
  const float pos = __fmul_rn(__fmul_rn(alpha, __fmul_rn(q, q)), -ls_pos);
  return __fsub_rn(pos, neg);
}

__device__ __forceinline__ float pair_cost(const float4 pb, const Corners& pc, const float4 tb,
                                           const Corners& tc, float class_cost,
                                           const CostArgs& a) {
  // torch.cdist(p=1) over the four cxcywh coordinates (kernels_matcher.py:98-103)
  const float l1 = __fadd_rn(
      __fadd_rn(__fadd_rn(fabsf(__fsub_rn(pb.x, tb.x)), fabsf(__fsub_rn(pb.y, tb.y))),
                fabsf(__fsub_rn(pb.z, tb.z))),
      fabsf(__fsub_rn(pb.w, tb.w)));
  // GIoU with clamped union and hull (kernels_matcher.py:118-127)
  const float iw = __fsub_rn(fminf(pc.x1, tc.x1), fmaxf(pc.x0, tc.x0));
  const float ih = __fsub_rn(fminf(pc.y1, tc.y1), fmaxf(pc.y0, tc.y0));
  const float inter = __fmul_rn(fmaxf(iw, 0.0f), fmaxf(ih, 0.0f));
  const float uni = __fsub_rn(__fadd_rn(pc.area, tc.area), inter);
  const float iou = __fdiv_rn(inter, fmaxf(uni, kBoxEps));
  const float ew = __fsub_rn(fmaxf(pc.x1, tc.x1), fminf(pc.x0, tc.x0));
  const float eh = __fsub_rn(fmaxf(pc.y1, tc.y1), fminf(pc.y0, tc.y0));
  const float hull = __fmul_rn(fmaxf(ew, 0.0f), fmaxf(eh, 0.0f));
  const float giou = __fsub_rn(iou, __fdiv_rn(__fsub_rn(hull, uni), fmaxf(hull, kBoxEps)));
  // cost_bbox * l1 + cost_class * class + cost_giou * (-giou)  (kernels_matcher.py:264)
  return __fadd_rn(__fadd_rn(__fmul_rn(a.w_bbox, l1), __fmul_rn(a.w_class, class_cost)),
                   __fmul_rn(a.w_giou, -giou));
}

// Largest image b with offsets[b] <= col (images with no targets are skipped).
__device__ __forceinline__ int image_of(const int32_t* offsets, int B, int col) {
  int lo = 0, hi = B;
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

template <bool kVec>
__global__ void __launch_bounds__(kThreads) cost_kernel(const CostArgs a) {
  const int64_t col0 = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (col0 >= a.ld) return;
  const int layer = blockIdx.z;
  const int q_begin = blockIdx.y * a.rows_per_cta;
  const int q_end = min(a.Q, q_begin + a.rows_per_cta);

  float4 tb[4];
  Corners tc[4];
  int label[4], image[4];
  bool valid[4];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int64_t col = col0 + c;
    valid[c] = col < a.S;
    if (valid[c]) {
      image[c] = image_of(a.offsets, a.B, static_cast<int>(col));
      tb[c] = __ldg(a.tboxes + col);
      const int64_t raw = __ldg(a.labels + col);
      label[c] = static_cast<int>(raw < 0 ? 0 : (raw >= a.C ? a.C - 1 : raw));
      tc[c] = corners(tb[c]);
    } else {
      image[c] = 0;
      label[c] = 0;
      tb[c] = make_float4(0.f, 0.f, 0.f, 0.f);
      tc[c] = Corners{0.f, 0.f, 0.f, 0.f, 0.f};
    }
  }
  const int64_t layer_base = static_cast<int64_t>(layer) * a.B;

  for (int q = q_begin + threadIdx.y; q < q_end; q += blockDim.y) {
    float r[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      r[c] = 0.0f;
      if (valid[c]) {
        const int64_t pq = (layer_base + image[c]) * a.Q + q;
        const float4 pb = __ldg(a.pboxes + pq);
        const float x = __ldg(a.logits + pq * a.C + label[c]);
        r[c] = pair_cost(pb, corners(pb), tb[c], tc[c], focal_cost(x, a.alpha, a.one_minus_alpha),
                         a);
      }
    }
    float* dst = a.out + (static_cast<int64_t>(layer) * a.Q + q) * a.ld + col0;
    if (kVec) {
      *reinterpret_cast<float4*>(dst) = make_float4(r[0], r[1], r[2], r[3]);
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        if (col0 + c < a.ld) dst[c] = r[c];
      }
    }
  }
}

}  // namespace
}  // namespace rfm

extern "C" int rfm_cost(const float* pred_logits, const float* pred_boxes,
                        const int64_t* tgt_labels, const float* tgt_boxes,
                        const int32_t* tgt_offsets, int num_layers, int num_images,
                        int num_queries, int num_classes, int sum_targets, int64_t ld,
                        float cost_class, float cost_bbox, float cost_giou, float focal_alpha,
                        float* out, void* stream) {
  using namespace rfm;
  if (num_layers < 1 || num_layers > 65535 || num_images < 1 || num_queries < 1 ||
      num_classes < 1 || sum_targets < 0 || ld < sum_targets) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (ld == 0) return RFM_OK;
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
  a.one_minus_alpha = static_cast<float>(1.0 - static_cast<double>(focal_alpha));
  a.out = out;

  const int64_t chunks = (ld + 3) / 4;
  int tx = 1;
  while (tx < chunks && tx < 64) tx <<= 1;
  const int ty = kThreads / tx;
  a.rows_per_cta = ty * kRowsPerThread;
  const int64_t gx = (chunks + tx - 1) / tx;
  const int64_t gy = (num_queries + a.rows_per_cta - 1) / a.rows_per_cta;
  if (gx > 0x7fffffff || gy > 65535) return RFM_ERR_UNSUPPORTED;
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy),
                  static_cast<unsigned>(num_layers));
  const dim3 block(tx, ty, 1);
  if ((ld & 3) == 0 && aligned16(out)) {
    cost_kernel<true><<<grid, block, 0, as_stream(stream)>>>(a);
  } else {
    cost_kernel<false><<<grid, block, 0, as_stream(stream)>>>(a);
  }
  return launch_status();
}
