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
// of value, and the D outputs are one coalesced store.  The backward warp
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

template <bool kBackward>
__global__ void __launch_bounds__(32 * kMsdaWarps) msda_kernel(const MsdaArgs a) {
  __shared__ int s_h[kMsdaMaxLevels], s_w[kMsdaMaxLevels];
  __shared__ int64_t s_start[kMsdaMaxLevels];
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
  const int64_t task = static_cast<int64_t>(blockIdx.x) * kMsdaWarps + (threadIdx.x >> 5);
  const int64_t tasks = static_cast<int64_t>(a.B) * a.Q * a.M;
  if (task >= tasks) return;
  const int m = static_cast<int>(task % a.M);
  const int64_t bq = task / a.M;
  const int b = static_cast<int>(bq / a.Q);
  const int LP = a.L * a.P;
  const float* loc = a.loc + task * LP * 2;
  const float* wts = a.w + task * LP;
  // value row (s) of head m of image b starts at ((b * S + s) * M + m) * D
  const int64_t row_stride = static_cast<int64_t>(a.M) * a.D;
  const float* vb = a.value + (static_cast<int64_t>(b) * a.S * a.M + m) * a.D;
  for (int d0 = 0; d0 < a.D; d0 += 32) {
    const int d = d0 + lane;
    const bool on = d < a.D;
    float acc = 0.0f;
    const float g = (kBackward && on) ? a.grad_out[task * a.D + d] : 0.0f;
    for (int l = 0; l < a.L; ++l) {
      const int H = s_h[l], W = s_w[l];
      const float* vl = vb + s_start[l] * row_stride;
      for (int p = 0; p < a.P; ++p) {
        const int sp = l * a.P + p;
        const float lx = __ldg(loc + 2 * sp), ly = __ldg(loc + 2 * sp + 1);
        const float ws = __ldg(wts + sp);
        const Corners4 c = corners_of(lx, ly, H, W);
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = (on && c.idx[k] >= 0) ? __ldg(vl + c.idx[k] * row_stride + d) : 0.0f;
        const float sample = ((c.wt[0] * v[0] + c.wt[1] * v[1]) + c.wt[2] * v[2]) + c.wt[3] * v[3];
        if (!kBackward) {
          acc += ws * sample;
        } else {
          // d sample / dx and / dy (pixel units), then / dloc = * W and * H
          const float gx = 1.0f - c.fx, gy = 1.0f - c.fy;
          const float dsx = gy * (v[1] - v[0]) + c.fy * (v[3] - v[2]);
          const float dsy = gx * (v[2] - v[0]) + c.fx * (v[3] - v[1]);
          const float gw = warp_sum(g * sample);
          const float glx = warp_sum(g * dsx) * ws * static_cast<float>(W);
          const float gly = warp_sum(g * dsy) * ws * static_cast<float>(H);
          if (lane == 0) {
            // channel passes (D > 32) accumulate into the same slots
            if (d0 == 0) {
              a.grad_w[task * LP + sp] = gw;
              a.grad_loc[(task * LP + sp) * 2] = glx;
              a.grad_loc[(task * LP + sp) * 2 + 1] = gly;
            } else {
              a.grad_w[task * LP + sp] += gw;
              a.grad_loc[(task * LP + sp) * 2] += glx;
              a.grad_loc[(task * LP + sp) * 2 + 1] += gly;
            }
          }
          if (on) {
            const float gs = ws * g;
            float* gvl = a.grad_value + (static_cast<int64_t>(b) * a.S * a.M + m) * a.D + s_start[l] * row_stride;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              if (c.idx[k] >= 0) atomicAdd(gvl + c.idx[k] * row_stride + d, gs * c.wt[k]);
            }
          }
        }
      }
    }
    if (!kBackward && on) a.out[task * a.D + d] = acc;
  }
}

int msda_args(MsdaArgs& a, const float* value, const int64_t* shapes, const int64_t* start, const float* loc,
              const float* w, int B, int S, int M, int D, int Q, int L, int P) {
  if (B < 1 || S < 1 || M < 1 || D < 1 || Q < 0 || L < 1 || L > kMsdaMaxLevels || P < 1 || P > kMsdaMaxPoints ||
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
