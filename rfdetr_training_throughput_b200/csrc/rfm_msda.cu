// Multi-scale deformable attention (the decoder's and encoder's MSDeformAttn
// core), forward and backward, fp32.
//
// Replaces the core the reference routes to a prebuilt Deformable-DETR kernel
// (kernels_msda_cuda.py: DeformableAttention, deformable_attention,
// module_forward; patches fused_msda / fused_msda_native, patches.py:566-635),
// written from the published sampling rule of Deformable DETR
// (ms_deform_attn_core_pytorch: one F.grid_sample per level, bilinear,
// align_corners=False, zero padding, then the attention-weighted sum):
//
//   out[b, q, m, :] = sum_{l, p} w[b, q, m, l, p] * bilinear(V_l[b, :, :, m, :], loc[b, q, m, l, p])
//
// with V_l the level-l slice of value [B, S, M, D] (rows level_start[l] ..,
// H_l x W_l row-major), and the sample taken at pixel coordinates
// x = loc.x * W_l - 0.5, y = loc.y * H_l - 0.5: the four neighbours
// (floor(y) + {0,1}, floor(x) + {0,1}) weighted (1-fy)(1-fx), (1-fy)fx,
// fy(1-fx), fy fx, a neighbour outside the map contributing zero.
//
// Layout.  One warp computes one (b, q, m): lane d holds channel d (channels
// beyond 32 in further passes), so each neighbour is one coalesced 128-byte row
// of value, and the D outputs are one coalesced store.  The samples' neighbour
// rows and weights are worked out once per warp, lane j for sample j, and
// read by every lane from shared memory as broadcasts.  The backward warp
// recomputes the samples, reduces the gradients of the sampling location and of
// the attention weight over the channels with warp shuffles, and adds the
// value gradient into the four neighbours with atomic adds, each lane its own
// channel, so a neighbour's update is one coalesced 128-byte reduction per warp
// (samples of different queries may hit the same neighbour, hence atomics;
// the order of the additions, and so the last bits of grad_value, can vary
// from run to run, as with the reference kernel and grid_sample's backward).
#include "rfm_common.cuh"

namespace rfm {
namespace {

constexpr int kMsdaWarps = 8;
constexpr int kMsdaMaxLevels = 8;
constexpr int kMsdaMaxPoints = 16;
constexpr int kMsdaMaxPasses = 4;  // head_dim <= 128: up to four channel passes of 32 lanes

struct MsdaArgs {
  const float* value;    // [B, S, M, D]
  const int64_t* shapes; // [L, 2] (H, W)
  const int64_t* start;  // [L]
  const float* loc;      // [B, Q, M, L, P, 2]
  const float* w;        // [B, Q, M, L, P]
  int B, S, M, D, Q, L, P;
  float* out;            // [B, Q, M, D]
  const float* grad_out; // [B, Q, M, D]
  float* grad_value;     // [B, S, M, D] (accumulated into)
  float* grad_loc;       // [B, Q, M, L, P, 2]
  float* grad_w;         // [B, Q, M, L, P]
};

// The four neighbours of one sample: their row offsets within the level's
// value rows (-1 when outside the map) and bilinear weights, plus the
// fractional parts (for the location gradient).
struct Corners4 {
  int idx[4];
  float wt[4];
  float fx, fy;
};

__device__ __forceinline__ Corners4 corners_of(float lx, float ly, int H, int W) {
  Corners4 c;
  const float x = lx * static_cast<float>(W) - 0.5f;
  const float y = ly * static_cast<float>(H) - 0.5f;
  const float x0f = floorf(x), y0f = floorf(y);
  const int x0 = static_cast<int>(x0f), y0 = static_cast<int>(y0f);
  c.fx = x - x0f;
  c.fy = y - y0f;
  const float gx = 1.0f - c.fx, gy = 1.0f - c.fy;
  const bool in_x0 = x0 >= 0 && x0 < W, in_x1 = x0 + 1 >= 0 && x0 + 1 < W;
  const bool in_y0 = y0 >= 0 && y0 < H, in_y1 = y0 + 1 >= 0 && y0 + 1 < H;
  c.idx[0] = (in_y0 && in_x0) ? y0 * W + x0 : -1;
  c.idx[1] = (in_y0 && in_x1) ? y0 * W + x0 + 1 : -1;
  c.idx[2] = (in_y1 && in_x0) ? (y0 + 1) * W + x0 : -1;
  c.idx[3] = (in_y1 && in_x1) ? (y0 + 1) * W + x0 + 1 : -1;
  c.wt[0] = gy * gx;
  c.wt[1] = gy * c.fx;
  c.wt[2] = c.fy * gx;
  c.wt[3] = c.fy * c.fx;
  return c;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFullMask, v, o);
  return v;
}

// One sample's neighbours as the warp's lanes read them (64 bytes, four
// 16-byte broadcasts): value rows (within the (b, m) plane, -1 outside) and
// bilinear weights, and for the backward pass the attention weight, the
// fractional position and the map size.
struct SampleSlot {
  int4 idx;
  float4 wt;     // forward: attention weight x bilinear weight; backward: bilinear weight
  float4 extra;  // ws, fx, fy, W
  float4 extra2; // H
};

template <bool kBackward>
__global__ void __launch_bounds__(32 * kMsdaWarps) msda_kernel(const MsdaArgs a) {
  __shared__ int s_h[kMsdaMaxLevels], s_w[kMsdaMaxLevels];
  __shared__ int64_t s_start[kMsdaMaxLevels];
  __shared__ SampleSlot s_slot[kMsdaWarps][32];
  if (threadIdx.x < a.L) {
    // a level whose rows do not lie inside [0, S) is sampled as empty (every
    // neighbour outside the map), so no access leaves the value tensor
    const int64_t h = a.shapes[2 * threadIdx.x], w = a.shapes[2 * threadIdx.x + 1];
    const int64_t st = a.start[threadIdx.x];
    const bool ok = h > 0 && w > 0 && h <= 65536 && w <= 65536 && st >= 0 && st + h * w <= a.S;
    s_h[threadIdx.x] = ok ? static_cast<int>(h) : 0;
    s_w[threadIdx.x] = ok ? static_cast<int>(w) : 0;
    s_start[threadIdx.x] = ok ? st : 0;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t task = static_cast<int64_t>(blockIdx.x) * kMsdaWarps + warp;
  const int64_t tasks = static_cast<int64_t>(a.B) * a.Q * a.M;
  if (task >= tasks) return;
  const int m = static_cast<int>(task % a.M);
  const int b = static_cast<int>(task / a.M / a.Q);
  const int LP = a.L * a.P;
  const int passes = (a.D + 31) >> 5;  // <= kMsdaMaxPasses channel passes of 32
  // value row s of head m of image b: value + ((b * S + s) * M + m) * D
  const int64_t row_stride = static_cast<int64_t>(a.M) * a.D;
  const float* vb = a.value + (static_cast<int64_t>(b) * a.S * a.M + m) * a.D;
  float* gvb = kBackward ? a.grad_value + (static_cast<int64_t>(b) * a.S * a.M + m) * a.D : nullptr;
  float acc[kMsdaMaxPasses], g[kMsdaMaxPasses];
#pragma unroll
  for (int c = 0; c < kMsdaMaxPasses; ++c) {
    acc[c] = 0.0f;
    const int d = 32 * c + lane;
    g[c] = (kBackward && c < passes && d < a.D) ? a.grad_out[task * a.D + d] : 0.0f;
  }
  SampleSlot* slot = s_slot[warp];
  for (int c0 = 0; c0 < LP; c0 += 32) {
    // lane j prepares sample c0 + j
    const int sp = c0 + lane;
    if (sp < LP) {
      const int l = sp / a.P;
      const int H = s_h[l], W = s_w[l];
      const float lx = __ldg(a.loc + 2 * (task * LP + sp)), ly = __ldg(a.loc + 2 * (task * LP + sp) + 1);
      const float ws = __ldg(a.w + task * LP + sp);
      const Corners4 c = corners_of(lx, ly, H, W);
      SampleSlot sl;
      const int64_t st = s_start[l];
      sl.idx = make_int4(c.idx[0] < 0 ? -1 : static_cast<int>(st + c.idx[0]),
                         c.idx[1] < 0 ? -1 : static_cast<int>(st + c.idx[1]),
                         c.idx[2] < 0 ? -1 : static_cast<int>(st + c.idx[2]),
                         c.idx[3] < 0 ? -1 : static_cast<int>(st + c.idx[3]));
      const float f = kBackward ? 1.0f : ws;
      sl.wt = make_float4(f * c.wt[0], f * c.wt[1], f * c.wt[2], f * c.wt[3]);
      sl.extra = make_float4(ws, c.fx, c.fy, static_cast<float>(W));
      sl.extra2 = make_float4(static_cast<float>(H), 0.f, 0.f, 0.f);
      slot[lane] = sl;
    }
    __syncwarp();
    const int n = min(32, LP - c0);
    for (int j = 0; j < n; ++j) {
      const int4 ix = slot[j].idx;
      const float4 wt = slot[j].wt;
      float gw = 0.f, gx = 0.f, gy = 0.f;  // backward: this lane's channels' shares
      float ws = 0.f, fx = 0.f, fy = 0.f;
      if (kBackward) {
        const float4 e = slot[j].extra;
        ws = e.x;
        fx = e.y;
        fy = e.z;
      }
#pragma unroll
      for (int c = 0; c < kMsdaMaxPasses; ++c) {
        const int d = 32 * c + lane;
        if (c >= passes) break;
        const bool on = d < a.D;
        const float v0 = (on && ix.x >= 0) ? __ldg(vb + ix.x * row_stride + d) : 0.0f;
        const float v1 = (on && ix.y >= 0) ? __ldg(vb + ix.y * row_stride + d) : 0.0f;
        const float v2 = (on && ix.z >= 0) ? __ldg(vb + ix.z * row_stride + d) : 0.0f;
        const float v3 = (on && ix.w >= 0) ? __ldg(vb + ix.w * row_stride + d) : 0.0f;
        const float sample = ((wt.x * v0 + wt.y * v1) + wt.z * v2) + wt.w * v3;
        if (!kBackward) {
          acc[c] += sample;
        } else {
          const float hx = 1.0f - fx, hy = 1.0f - fy;
          gw += g[c] * sample;
          gx += g[c] * (hy * (v1 - v0) + fy * (v3 - v2));
          gy += g[c] * (hx * (v2 - v0) + fx * (v3 - v1));
          if (on) {
            const float gs = ws * g[c];
            if (ix.x >= 0) atomicAdd(gvb + ix.x * row_stride + d, gs * wt.x);
            if (ix.y >= 0) atomicAdd(gvb + ix.y * row_stride + d, gs * wt.y);
            if (ix.z >= 0) atomicAdd(gvb + ix.z * row_stride + d, gs * wt.z);
            if (ix.w >= 0) atomicAdd(gvb + ix.w * row_stride + d, gs * wt.w);
          }
        }
      }
      if (kBackward) {
        // sums over the channels: d out / d w, and d out / d loc = w * d sample / d (x, y) * (W, H)
        gw = warp_sum(gw);
        gx = warp_sum(gx);
        gy = warp_sum(gy);
        if (lane == 0) {
          const int64_t k = task * LP + c0 + j;
          a.grad_w[k] = gw;
          a.grad_loc[2 * k] = gx * ws * slot[j].extra.w;
          a.grad_loc[2 * k + 1] = gy * ws * slot[j].extra2.x;
        }
      }
    }
    __syncwarp();  // every lane is done with the slots before the next chunk rewrites them
  }
  if (!kBackward) {
#pragma unroll
    for (int c = 0; c < kMsdaMaxPasses; ++c) {
      const int d = 32 * c + lane;
      if (c < passes && d < a.D) a.out[task * a.D + d] = acc[c];
    }
  }
}

int msda_args(MsdaArgs& a, const float* value, const int64_t* shapes, const int64_t* start, const float* loc,
              const float* w, int B, int S, int M, int D, int Q, int L, int P) {
  if (B < 1 || S < 1 || M < 1 || D < 1 || D > 32 * kMsdaMaxPasses || Q < 0 || L < 1 || L > kMsdaMaxLevels ||
      P < 1 || P > kMsdaMaxPoints || static_cast<int64_t>(S) * M * D > 0x7fffffff ||
      value == nullptr || shapes == nullptr || start == nullptr ||
      (Q > 0 && (loc == nullptr || w == nullptr))) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  if (static_cast<int64_t>(B) * Q * M > (int64_t(1) << 36)) return RFM_ERR_UNSUPPORTED;
  a.value = value;
  a.shapes = shapes;
  a.start = start;
  a.loc = loc;
  a.w = w;
  a.B = B;
  a.S = S;
  a.M = M;
  a.D = D;
  a.Q = Q;
  a.L = L;
  a.P = P;
  a.out = nullptr;
  a.grad_out = nullptr;
  a.grad_value = nullptr;
  a.grad_loc = nullptr;
  a.grad_w = nullptr;
  return RFM_OK;
}

int64_t msda_blocks(const MsdaArgs& a) {
  return (static_cast<int64_t>(a.B) * a.Q * a.M + kMsdaWarps - 1) / kMsdaWarps;
}

}  // namespace
}  // namespace rfm

extern "C" int rfm_msda_forward(const float* value, const int64_t* spatial_shapes, const int64_t* level_start,
                                const float* sampling_locations, const float* attention_weights, int batch,
                                int sequence, int heads, int head_dim, int queries, int levels, int points,
                                float* out, void* stream) {
  using namespace rfm;
  MsdaArgs a;
  const int rc = msda_args(a, value, spatial_shapes, level_start, sampling_locations, attention_weights, batch,
                           sequence, heads, head_dim, queries, levels, points);
  if (rc != RFM_OK) return rc;
  if (queries == 0) return RFM_OK;
  if (out == nullptr) return RFM_ERR_INVALID_ARGUMENT;
  a.out = out;
  const int64_t blocks = msda_blocks(a);
  if (blocks > 0x7fffffff) return RFM_ERR_UNSUPPORTED;
  msda_kernel<false><<<static_cast<unsigned>(blocks), 32 * kMsdaWarps, 0, as_stream(stream)>>>(a);
  return launch_status();
}

extern "C" int rfm_msda_backward(const float* value, const int64_t* spatial_shapes, const int64_t* level_start,
                                 const float* sampling_locations, const float* attention_weights,
                                 const float* grad_out, int batch, int sequence, int heads, int head_dim,
                                 int queries, int levels, int points, float* grad_value, float* grad_locations,
                                 float* grad_weights, void* stream) {
  using namespace rfm;
  MsdaArgs a;
  const int rc = msda_args(a, value, spatial_shapes, level_start, sampling_locations, attention_weights, batch,
                           sequence, heads, head_dim, queries, levels, points);
  if (rc != RFM_OK) return rc;
  if (queries == 0) return RFM_OK;
  if (grad_out == nullptr || grad_value == nullptr || grad_locations == nullptr || grad_weights == nullptr) {
    return RFM_ERR_INVALID_ARGUMENT;
  }
  a.grad_out = grad_out;
  a.grad_value = grad_value;
  a.grad_loc = grad_locations;
  a.grad_w = grad_weights;
  const int64_t blocks = msda_blocks(a);
  if (blocks > 0x7fffffff) return RFM_ERR_UNSUPPORTED;
  msda_kernel<true><<<static_cast<unsigned>(blocks), 32 * kMsdaWarps, 0, as_stream(stream)>>>(a);
  return launch_status();
}
