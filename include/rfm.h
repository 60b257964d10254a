/*
 * rfm.h - C ABI of the B200 (sm_100a) Hungarian-matching library for RF-DETR.
 *
 * The library replaces the two device stages of RF-DETR's HungarianMatcher:
 *
 *   rfm_cost   builds the compact detection cost matrix in one pass
 *              (focal class cost, L1 box distance, GIoU, weighted sum).
 *              Replaces the Triton launcher fused_matcher_cost
 *              (kernels_matcher.py:179-234) as called by the patched
 *              HungarianMatcher._compute_compact_detection_cost_matrix
 *              (patches.py:123-149).
 *
 *   rfm_lsap   solves a batch of rectangular linear assignment problems read
 *              in place from that matrix (one warp per problem for large
 *              batches; a CTA of two or four warps per problem when the batch
 *              runs in one wave), with the exact arithmetic and tie-breaking of
 *              SciPy's rectangular_lsap, and
 *              writes the (query, target) index pairs straight into their
 *              final packed position. Replaces batch_lap / lsap_kernel
 *              (kernels_lap.py:271-305, :332-355) together with the device
 *              unpack of the patched _assign_padded (patches.py:379-418).
 *
 *   rfm_match  rfm_cost (target-major) then rfm_lsap in one call, the two
 *              kernels overlapped at their boundary: what the fused matcher
 *              step (HungarianMatcher.forward) runs.
 *
 *   rfm_lsap_dense  the same solver under the torch_linear_assignment
 *              contract: cost [P, W, T] -> matching [P, W] (task or -1).
 *              Replaces batch_lap (kernels_lap.py:332-355) behind the
 *              cuda_lap patch (patches.py:291-327).
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are DEVICE pointers owned by the caller, except
 *     where a comment says "host".  No entry point allocates device memory,
 *     synchronises the stream or the device, or copies to the host, except
 *     the setup calls of the sharded sweep's exchange (rfm_peer_alloc,
 *     rfm_peer_free, rfm_pair_push_store), which say so.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL is
 *     the legacy default stream) on the current device.
 *   - The return value reports argument and launch errors synchronously
 *     (RFM_OK on success); rfm_error_string() names it.  Per-problem numeric
 *     outcomes (infeasible or invalid costs) are written to the optional
 *     device `status` array and are only visible after the stream completes.
 *   - Calls are thread-compatible: concurrent calls on different streams are
 *     safe as long as they write disjoint outputs.
 *   - Per-context state is cached under the CUDA context's unique id: the
 *     raised dynamic-shared-memory attribute of the solver kernels and the
 *     device address of rfm_lsap_dense_noalloc's scratch.  A context that is
 *     destroyed and recreated (cudaDeviceReset) gets both set up again on its
 *     first call.  Occupancy figures are memoised per device.
 *   - rfm_lsap reads its problem descriptors with ordinary stream ordering;
 *     only inside rfm_match, after this library's own cost kernel, does the
 *     solver start early (programmatic stream serialization).
 */
#ifndef RFM_H_
#define RFM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes -------------------------------------------------------- */
#define RFM_OK 0
#define RFM_ERR_INVALID_ARGUMENT 1 /* null pointer, negative size, bad stride */
#define RFM_ERR_UNSUPPORTED 2      /* outside the supported envelope */
#define RFM_ERR_LAUNCH 3           /* CUDA reported an error at launch */
#define RFM_ERR_NO_DEVICE 4        /* no usable CUDA device */

/* ---- per-problem status codes written by the solvers --------------------- */
#define RFM_STATUS_OK 0
#define RFM_STATUS_INFEASIBLE 1    /* no finite assignment (SciPy: "cost matrix is infeasible") */
#define RFM_STATUS_INVALID 2       /* NaN or -inf entry (SciPy: "matrix contains invalid numeric entries") */
#define RFM_STATUS_NO_SINK 3       /* augmenting search hit its column bound (never expected) */

/* Largest extent of the longer side of one assignment problem. */
#define RFM_MAX_COLS 1024

/*
 * One assignment problem, read in place from a row-major cost matrix.
 * Element (query q, target t) of problem p lives at
 *     cost[cost_offset + q * ld + t],  0 <= q < num_queries, 0 <= t < num_targets.
 * Its min(num_queries, num_targets) result pairs are written to
 *     query_out[out_offset + k], target_out[out_offset + k]
 * in SciPy's order (ascending query index), with query_base added to every
 * emitted query index (the group offset g * group_width of Group DETR).
 * scratch_offset is filled in by rfm_lsap_make_plan (-1: none needed).
 */
typedef struct rfm_problem {
  int64_t cost_offset;
  int64_t out_offset;
  int64_t scratch_offset;
  int32_t num_queries;
  int32_t num_targets;
  int32_t query_base;
  int32_t reserved; /* must be 0 */
} rfm_problem;

/*
 * Launch plan for one batch of problems, computed on the host from the
 * problem sizes (which the caller knows without reading the device) by
 * rfm_lsap_make_plan.  Treat it as opaque.
 */
typedef struct rfm_lsap_plan {
  int32_t cols_per_lane;    /* kernel instantiation: max(rows, cols) <= 32 * cols_per_lane */
  int32_t max_rows;         /* largest min(num_queries, num_targets) in the batch */
  int32_t num_problems;
  int32_t num_ctas;         /* entries of the CTA table */
  int32_t cta_smem_bytes;   /* dynamic shared memory of one CTA */
  int32_t tile_cap_floats;  /* largest cost tile staged on chip */
  int32_t flags;            /* RFM_PLAN_* */
  int32_t reserved;
  int64_t stride_q;         /* cost element (q, t) at cost_offset + q*stride_q + t*stride_t */
  int64_t stride_t;
  int64_t workspace_bytes;  /* device scratch rfm_lsap needs for this batch */
} rfm_lsap_plan;

/* rfm_lsap_plan.flags: the batch runs on persistent warps; warp w starts on
 * problem w, and the warps pull the rest in order from a counter kept at the
 * start of the workspace. */
#define RFM_PLAN_PERSISTENT 1

/* Layouts rfm_cost can write. */
#define RFM_LAYOUT_QUERY_MAJOR 0  /* out[l][q][ld]: the compact [Q, sum T] matrix of patches.py:149 */
#define RFM_LAYOUT_TARGET_MAJOR 1 /* out[l][col][ld]: its transpose, row = target, ld >= Q */

/* Library identification string (static storage). */
const char* rfm_version(void);

/* Human-readable name of a return code (static storage). */
const char* rfm_error_string(int code);

/*
 * Compact detection cost matrix for L decoder layers sharing one set of
 * targets:
 *
 *   out[l, q, off[b] + t] = cost_bbox  * L1(pred_box[l,b,q], tgt_box[off[b]+t])
 *                         + cost_class * focal(pred_logit[l,b,q,label[off[b]+t]])
 *                         + cost_giou  * -GIoU(xyxy(pred_box[l,b,q]), xyxy(tgt_box[off[b]+t]))
 *
 * for every layer l < num_layers, image b < num_images, query q < num_queries
 * and target t < off[b+1] - off[b].  Row q of the matrix holds image b's
 * targets in columns off[b] .. off[b+1]-1 and is evaluated against image b's
 * query q; this is the [Q, sum T] layout produced by
 * torch.cat([padded[b, :, :T_b] for b], -1) at patches.py:149.
 *
 *   pred_logits  [L, B, Q, C] float32, contiguous
 *   pred_boxes   [L, B, Q, 4] float32 cxcywh, contiguous, 16-byte aligned
 *   tgt_labels   [S] int64, clamped into [0, C-1] before use
 *                (kernels_matcher.py:133-134)
 *   tgt_boxes    [S, 4] float32 cxcywh, 16-byte aligned
 *   tgt_offsets  [B + 1] int32, off[0] = 0, off[B] = S = sum_targets
 *   layout       RFM_LAYOUT_QUERY_MAJOR: out [L, Q, ld], ld >= S, the compact
 *                matrix itself; RFM_LAYOUT_TARGET_MAJOR: out [L, S, ld],
 *                ld >= Q, ld % 4 == 0, its transpose (each target's row holds
 *                its image's Q queries), the layout the solver reads fastest.
 *   out          float32, 16-byte aligned for the target-major layout.  Pad
 *                columns (S .. ld-1, resp. Q .. ld-1) are written with 0.
 *                Query-major with ld % 4 == 0 and a 16-byte aligned `out`
 *                uses 128-bit stores; any other ld is accepted.
 *
 * Focal cost with gamma 2 (kernels_matcher.py:49-50, 257-260):
 *   p = sigmoid(x)
 *   focal(x) = alpha (1-p)^2 (-logsigmoid(x)) - (1-alpha) p^2 (-logsigmoid(-x))
 * GIoU with the 1e-7 clamps of kernels_matcher.py:121-127.
 */
int rfm_cost(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
             const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
             int num_queries, int num_classes, int sum_targets, int64_t ld, int layout,
             float cost_class, float cost_bbox, float cost_giou, float focal_alpha, float* out,
             void* stream);

/*
 * Host-side planning for rfm_lsap.  Reads the sizes of host_problems[0..n)
 * and the cost strides (element (q, t) of a problem at
 * cost_offset + q*stride_q + t*stride_t), writes each problem's
 * scratch_offset (floats into the workspace, or -1), fills the CTA table
 * host_ctas (4 int32 per CTA, room for num_problems entries; plan->num_ctas
 * are used) and *plan.  Problems are packed into CTAs in the order given, so
 * callers sort them by decreasing num_queries * num_targets for balance.
 * tile_cap_floats bounds the cost tile a problem may stage on chip (-1: the
 * library default, 0: never stage).  Pure host code: no CUDA call.
 */
int rfm_lsap_make_plan(rfm_problem* host_problems, int num_problems, int64_t stride_q,
                       int64_t stride_t, int64_t tile_cap_floats, int32_t* host_ctas,
                       rfm_lsap_plan* plan);

/*
 * Batched exact rectangular assignment with SciPy's semantics
 * (scipy.optimize.linear_sum_assignment, rectangular_lsap in SciPy 1.18.1):
 * the problem is solved untransposed when num_targets >= num_queries and
 * transposed (rows = targets) otherwise; duals and path costs are float64 on
 * the float32 costs, and ties between equal path costs are broken exactly as
 * SciPy's sequential scan breaks them.
 *
 *   cost        float32 matrix addressed by each problem's cost_offset and the
 *               plan's strides
 *   problems    [num_problems] DEVICE copy of the planned rfm_problem array
 *   ctas        [plan->num_ctas * 4] DEVICE copy of the planned CTA table
 *   plan        host pointer to the plan rfm_lsap_make_plan returned
 *   query_out,
 *   target_out  int64 outputs addressed by out_offset
 *   status      [num_problems] int32 RFM_STATUS_* or NULL
 *   workspace   device scratch of plan->workspace_bytes bytes (NULL if 0)
 *
 * Problems whose smaller side is 0 write nothing.  When a problem's status
 * is not RFM_STATUS_OK its output slots are filled with -1.
 */
int rfm_lsap(const float* cost, const rfm_problem* problems, const int32_t* ctas,
             const rfm_lsap_plan* plan, int64_t* query_out, int64_t* target_out, int32_t* status,
             void* workspace, void* stream);

/*
 * The whole matcher step in one call: rfm_cost into the target-major `cost`
 * ([num_layers, sum_targets, ld]) followed by rfm_lsap on it, with the same
 * arguments and results as those two calls.  No counterpart in the reference
 * (whose step is the Triton cost kernel, a padded copy and the solver launched
 * separately, patches.py:123-149,379-418).  The plan must have been made for
 * that matrix (stride_q 1, stride_t ld).  With a persistent plan the cost
 * kernel resets the solver's counter in `workspace`, so no memset runs between
 * the kernels, and the solver is launched with programmatic stream
 * serialization: its CTAs start while the cost kernel finishes and wait for
 * its completion before they read the matrix.
 */
int rfm_match(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
              const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
              int num_queries, int num_classes, int sum_targets, int64_t ld, float cost_class,
              float cost_bbox, float cost_giou, float focal_alpha, float* cost,
              const rfm_problem* problems, const int32_t* ctas, const rfm_lsap_plan* plan,
              int64_t* query_out, int64_t* target_out, int32_t* status, void* workspace,
              void* stream);

/*
 * torch_linear_assignment.batch_linear_assignment contract
 * (kernels_lap.py:336-341): cost [P, W, T] float32 contiguous ->
 * matching [P, W] int64 with the task of each worker, -1 when unassigned.
 * Solved per problem with SciPy's semantics as in rfm_lsap.
 * `workspace` must hold rfm_lsap_dense_workspace_bytes(P, W, T) bytes: the
 * scratch of tiles that are staged off chip, and for batches of 512 or more
 * problems a 256-byte counter after it (the solver's CTAs may claim problems
 * from it; it is reset on the stream by every call).
 */
int64_t rfm_lsap_dense_workspace_bytes(int num_problems, int num_workers, int num_tasks);
int rfm_lsap_dense(const float* cost, int num_problems, int num_workers, int num_tasks,
                   int64_t* matching, int32_t* status, void* workspace, void* stream);

/*
 * rfm_lsap_dense without a caller-provided workspace.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory where
 * they call the solver (a C FFI host without a device allocator, or a training
 * step that must not add a cudaMalloc/cudaFree or compete with the
 * framework's caching allocator).  The scratch is a built-in device array of
 * RFM_NOALLOC_SCRATCH_BYTES held by every GPU that loads the library.
 *
 *   - Same inputs, outputs and results as rfm_lsap_dense; allocates nothing.
 *   - Returns RFM_ERR_UNSUPPORTED, without launching, when the batch needs more
 *     scratch than the built-in array (rfm_lsap_dense_workspace_bytes() >
 *     RFM_NOALLOC_SCRATCH_BYTES); use rfm_lsap_dense with a workspace then.
 *   - The first call in a CUDA context looks up the array's device address
 *     (once per device while its primary context lives, again after the
 *     context is destroyed and recreated); make that first call before any
 *     stream capture.
 *   - All calls share the array: calls whose GPU work overlaps (e.g. on two
 *     streams at once) race on it.  Nothing in it needs clearing between calls.
 */
#define RFM_NOALLOC_SCRATCH_BYTES (16u << 20)
int rfm_lsap_dense_noalloc(const float* cost, int num_problems, int num_workers, int num_tasks,
                           int64_t* matching, int32_t* status, void* stream);

/*
 * Matched-box losses of the DETR-family criterion (SetCriterion.loss_boxes, the
 * consumer of the matcher's indices: criterion.py:904/906 as cited at
 * patches.py:339-341), read from the packed pairs rfm_lsap writes.  For every
 * pair k of (layer l, image b) — query_idx[k], target_idx[k] for k in
 * [pair_offsets[l*B + b], pair_offsets[l*B + b + 1]) — with p = pred_boxes[l, b, q]
 * and t = tgt_boxes[off[b] + target] (cxcywh):
 *
 *   l1_part[l*B + b]   = sum_k |p - t|_1                         (4 coordinates)
 *   giou_part[l*B + b] = sum_k (1 - GIoU(xyxy(p), xyxy(t)))       (unclamped GIoU)
 *
 * summed in a fixed order (deterministic).  Pairs holding -1 (an unsolved
 * problem) or an index outside their image are skipped.  The caller sums the
 * parts per layer and normalises by the number of boxes.
 *
 *   pred_boxes   [L, B, Q, 4] float32, 16-byte aligned
 *   tgt_boxes    [S, 4] float32, 16-byte aligned; tgt_offsets [B + 1] int32
 *   query_idx, target_idx  int64 pairs; pair_offsets [L*B + 1] int32
 *
 * rfm_box_loss_backward writes d/dpred of sum_l (grad_l1[l] * l1[l] +
 * grad_giou[l] * giou[l]) into grad_pred [L, B, Q, 4] at every matched query's
 * box (the caller zeroes the other entries); grad_l1, grad_giou are [L] device
 * arrays.  Gradients follow torch's autograd of the same expressions (ties of
 * min/max split evenly, clamp(min=0) passes at 0, |x| has slope sign(x)).
 * No counterpart kernel in the reference.
 */
int rfm_box_loss_forward(const float* pred_boxes, const float* tgt_boxes, const int32_t* tgt_offsets,
                         const int64_t* query_idx, const int64_t* target_idx, const int32_t* pair_offsets,
                         int num_layers, int num_images, int num_queries, int sum_targets, float* l1_part,
                         float* giou_part, void* stream);
int rfm_box_loss_backward(const float* pred_boxes, const float* tgt_boxes, const int32_t* tgt_offsets,
                          const int64_t* query_idx, const int64_t* target_idx, const int32_t* pair_offsets,
                          int num_layers, int num_images, int num_queries, int sum_targets,
                          const float* grad_l1, const float* grad_giou, float* grad_pred, void* stream);

/*
 * Classification loss of the DETR-family criterion (SetCriterion.loss_labels,
 * the criterion's other consumer of the matcher's indices: the target-class
 * scatter at criterion.py:562 as cited at patches.py:339-341), evaluated over
 * every logit with the matched (query, class) slots as positives, read from the
 * packed pairs rfm_lsap writes (same pair layout as rfm_box_loss_forward).
 * For every logit x = pred_logits[l, b, q, c], p = sigmoid(x), softplus(x) =
 * log(1 + exp(x)), and y = 1 exactly when query q of (l, b) is matched to a
 * target whose label is c:
 *
 *   RFM_LABEL_LOSS_FOCAL   sigmoid focal loss, gamma 2 (Deformable DETR):
 *       y = 1: alpha (1-p)^2 softplus(-x)     y = 0: (1-alpha) p^2 softplus(x)
 *   RFM_LABEL_LOSS_IA_BCE  IoU-aware BCE (LW-DETR, RF-DETR's criterion): with
 *       u = IoU(pred_boxes[l,b,q], its target box) (inter / union, unclamped)
 *       and t = max(p^alpha u^(1-alpha), 0.01) held constant:
 *       y = 1: (1-t) x + softplus(-x)          y = 0: p^2 softplus(x)
 *
 * loss_part receives rfm_label_loss_parts(L, B, Q, C) partial sums, (l, b)
 * major, each over a tile of about RFM_LABEL_LOSS_PART_ELEMS logits (a multiple
 * of 32 queries, 64 to 4096), each reduced in a fixed order; the caller
 * sums the parts of layer l (l * B * tiles .. (l+1) * B * tiles) and divides by
 * num_boxes.  correct_part (optional) counts matched queries whose largest
 * logit (smallest index among equal maxima) is their target's class, for the
 * criterion's class_error.  Matched labels outside [0, C) make no positive;
 * a query appears in at most one pair per (layer, image), as the matcher's
 * pairs guarantee.
 * A matched pair whose boxes both have zero area has IoU 0/0 = NaN, and the
 * IoU-aware loss is then NaN, as the unfused formula gives (clamp keeps NaN).
 * pred_boxes and tgt_boxes are read by the IoU-aware loss only (16-byte
 * aligned).  rfm_label_loss_backward writes grad_loss[l] * d(loss)/dx into
 * every element of grad_logits [L, B, Q, C] (torch's autograd of the same
 * expressions, t constant).  No counterpart kernel in the reference.
 */
#define RFM_LABEL_LOSS_FOCAL 0
#define RFM_LABEL_LOSS_IA_BCE 1
#define RFM_LABEL_LOSS_PART_ELEMS 8192
int64_t rfm_label_loss_parts(int num_layers, int num_images, int num_queries, int num_classes);
int rfm_label_loss_forward(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                           const float* tgt_boxes, const int32_t* tgt_offsets, const int64_t* query_idx,
                           const int64_t* target_idx, const int32_t* pair_offsets, int num_layers,
                           int num_images, int num_queries, int num_classes, int sum_targets, int mode,
                           float focal_alpha, float* loss_part, int32_t* correct_part, void* stream);
int rfm_label_loss_backward(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                            const float* tgt_boxes, const int32_t* tgt_offsets, const int64_t* query_idx,
                            const int64_t* target_idx, const int32_t* pair_offsets, int num_layers,
                            int num_images, int num_queries, int num_classes, int sum_targets, int mode,
                            float focal_alpha, const float* grad_loss, float* grad_logits, void* stream);

/*
 * Multi-scale deformable attention core (MSDeformAttn), fp32.  Replaces the
 * prebuilt Deformable-DETR kernel the reference routes the decoder and encoder
 * through (kernels_msda_cuda.py DeformableAttention.forward/backward: the
 * ms_deform_attn_forward / _backward calls, patches fused_msda and
 * fused_msda_native, patches.py:566-635); the arithmetic follows Deformable
 * DETR's published sampling rule (F.grid_sample, bilinear, align_corners=False,
 * zero padding, per level, then the attention-weighted sum):
 *
 *   out[b, q, m, :] = sum_{l, p} w[b, q, m, l, p] *
 *                     bilinear(value[b, start[l] + (y, x), m, :] at
 *                              x = loc[.., 0] * W_l - 0.5, y = loc[.., 1] * H_l - 0.5)
 *
 *   value               [B, S, M, D] float32 (sequence S = sum of H_l * W_l)
 *   spatial_shapes      [L, 2] int64 (H_l, W_l), DEVICE; level_start [L] int64
 *   sampling_locations  [B, Q, M, L, P, 2] float32 in [0, 1] (x, y)
 *   attention_weights   [B, Q, M, L, P] float32
 *   out                 [B, Q, M, D] float32 (= [B, Q, M * D])
 *
 * L <= 8, P <= 16, D <= 128, S * M * D < 2^31.  rfm_msda_backward adds
 * d out / d value (for grad_out) into
 * grad_value (the caller zeroes it; atomic adds, so its last bits may vary
 * between runs) and writes grad_locations [B, Q, M, L, P, 2] and grad_weights
 * [B, Q, M, L, P].
 */
int rfm_msda_forward(const float* value, const int64_t* spatial_shapes, const int64_t* level_start,
                     const float* sampling_locations, const float* attention_weights, int batch, int sequence,
                     int heads, int head_dim, int queries, int levels, int points, float* out, void* stream);
int rfm_msda_backward(const float* value, const int64_t* spatial_shapes, const int64_t* level_start,
                      const float* sampling_locations, const float* attention_weights, const float* grad_out,
                      int batch, int sequence, int heads, int head_dim, int queries, int levels, int points,
                      float* grad_value, float* grad_locations, float* grad_weights, void* stream);

/*
 * ---- The sharded sweep's exchange: pairs pushed into every rank's memory ----
 *
 * No counterpart in the reference, which matches on one GPU.  A batch split by
 * image over R ranks (one process per GPU) needs every rank's pairs on every
 * rank.  Instead of a separate all-gather, the solver's epilogue writes each
 * pair it produces into each rank's gathered buffer (peer memory over NVLink,
 * mapped into this process with CUDA IPC; plain stores, no multicast), so the
 * transfer overlaps the solve problem by problem.  A one-warp kernel then
 * raises this rank's flag on every rank and waits (bounded) for every rank's
 * flag.  Each gathered buffer is double-buffered by step parity, so a rank
 * that runs ahead writes the buffer of the step after the one its peers may
 * still be reading.
 */
#define RFM_MAX_PUSH 8

/*
 * Destinations that also receive every pair of rfm_lsap_push / rfm_match_push.
 * Pair k of a problem goes to query_out[d][o + k] and target_out[d][o + k] for
 * each d < count, with o = out_offset + (*epoch & 1) * parity_stride.  The
 * solver reads the list from device memory (rfm_pair_push_store puts it there),
 * so a captured launch picks up a list stored after the capture.
 */
typedef struct rfm_pair_push {
  int32_t count;                     /* destinations, 0..RFM_MAX_PUSH */
  int32_t reserved;                  /* must be 0 */
  int64_t parity_stride;             /* int64 elements between a destination's two buffers */
  const uint32_t* epoch;             /* DEVICE step counter of this rank (rfm_peer_sync advances it) */
  int64_t* query_out[RFM_MAX_PUSH];  /* DEVICE (peer-mapped) pointers */
  int64_t* target_out[RFM_MAX_PUSH];
} rfm_pair_push;

/* Checks `push` on the host and copies it to device_dst (DEVICE, 16-byte
 * aligned, sizeof(rfm_pair_push) bytes), synchronously. */
int rfm_pair_push_store(const rfm_pair_push* push, void* device_dst);

/* rfm_lsap / rfm_match whose pairs also go to the destinations of the push
 * list at device_push (DEVICE, stored by rfm_pair_push_store; NULL: none).
 * Pair plans only; dense batches are not pushed. */
int rfm_lsap_push(const float* cost, const rfm_problem* problems, const int32_t* ctas,
                  const rfm_lsap_plan* plan, int64_t* query_out, int64_t* target_out, int32_t* status,
                  void* workspace, const rfm_pair_push* device_push, void* stream);
int rfm_match_push(const float* pred_logits, const float* pred_boxes, const int64_t* tgt_labels,
                   const float* tgt_boxes, const int32_t* tgt_offsets, int num_layers, int num_images,
                   int num_queries, int num_classes, int sum_targets, int64_t ld, float cost_class,
                   float cost_bbox, float cost_giou, float focal_alpha, float* cost,
                   const rfm_problem* problems, const int32_t* ctas, const rfm_lsap_plan* plan,
                   int64_t* query_out, int64_t* target_out, int32_t* status, void* workspace,
                   const rfm_pair_push* device_push, void* stream);

/* Device memory another process on this node can map: `bytes` zeroed bytes on
 * the current device (*ptr), exportable through the 64-byte `handle`.  Free
 * with rfm_peer_free once every importer has closed it. */
int rfm_peer_alloc(int64_t bytes, void** ptr, unsigned char* handle);
/* Map another process's rfm_peer_alloc memory (its handle) into this one. */
int rfm_peer_open(const unsigned char* handle, void** ptr);
int rfm_peer_close(void* ptr);
int rfm_peer_free(void* ptr);

/*
 * One step's barrier across the ranks.  Every lane j < world stores
 * epoch + 1 into arrive[j] (this rank's flag on rank j, after a system-scope
 * fence that orders this GPU's earlier pushes before it), then waits until
 * flags[j] (rank j's flag on this rank) reaches epoch + 1, polling at most
 * spin_limit times; a wait that gives up sets *error to 1 and the kernel
 * returns.  *epoch is then advanced.
 */
typedef struct rfm_peer_sync_args {
  int32_t world;                   /* ranks, 1..RFM_MAX_PUSH */
  int32_t rank;
  int64_t spin_limit;              /* polls per wait, >= 1 */
  uint32_t* arrive[RFM_MAX_PUSH];  /* DEVICE (peer-mapped): this rank's flag word on rank j */
  const uint32_t* flags;           /* DEVICE: the world flag words of this rank */
  uint32_t* epoch;                 /* DEVICE: this rank's step counter */
  int32_t* error;                  /* DEVICE: set to 1 when a wait gives up */
} rfm_peer_sync_args;

int rfm_peer_sync(const rfm_peer_sync_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RFM_H_ */
