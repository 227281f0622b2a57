/*
 * frank_moe.h -- C ABI of the B200 (sm_100a) MoE FFN hot path.
 *
 * This library replaces three IREE-compiled components of frank-models:
 *   @moe_components.mul_mat_id      components/moe/mul_mat_id.mlir:22-120
 *   @moe_ffn_components.moe_ffn_block components/moe/moe_ffn_block.mlir:34-209
 *   @activation_components.swiglu   components/activation/swiglu.mlir:16-51
 * which the reference reaches through its test harness
 * (tests/utils.py:171-223, IREEModule.invoke / __getattr__) and, in MLIR,
 * from architectures/llm/transformer_layer_moe_prefill.mlir:216-224 and
 * transformer_layer_moe_decode.mlir:234-241.
 *
 * Conventions
 *  - Every pointer is a DEVICE pointer unless stated otherwise; the caller
 *    owns all buffers (inputs, outputs, workspace).  The library never
 *    allocates device memory.
 *  - Calls are asynchronous and ordered on the given CUDA stream
 *    (cudaStream_t passed as void*; NULL = legacy default stream).
 *  - Return 0 on success or a negative FRANK_E* code; frank_last_error()
 *    returns a thread-local message for the last failure on this thread.
 *  - Shapes follow the reference exactly:
 *      x        [T, H]      row-major                 (moe_ffn_block.mlir:35)
 *      wr       [E, H]      router weights            (moe_ffn_block.mlir:36)
 *      W_up/gate[F, H, E]   expert-innermost          (moe_ffn_block.mlir:37-38)
 *      W_down   [H, F, E]                             (moe_ffn_block.mlir:39)
 *      mul_mat_id weights [O, I, E], input [I, k, T], ids [k, T] int32,
 *      output [O, k, T]                               (mul_mat_id.mlir:23-26)
 *    Expert weights are consumed in a prepacked [E, O, I] layout made once
 *    by frank_prepack_experts (the reference re-transposes them on every
 *    call, mul_mat_id.mlir:38-48).
 */
#ifndef FRANK_MOE_H_
#define FRANK_MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define FRANK_F32 0
#define FRANK_BF16 1
/* router weights prepared once by frank_router_pack (a wr_dtype value) */
#define FRANK_ROUTER_PACKED 16

/* status codes */
#define FRANK_OK 0
#define FRANK_EINVAL (-1)   /* bad shape / dtype / pointer / alignment */
#define FRANK_EIDS (-2)     /* an expert id outside [0, E) */
#define FRANK_ECUDA (-3)    /* a CUDA runtime or driver call failed */
#define FRANK_ENOSPC (-4)   /* workspace smaller than *_workspace_size() */
#define FRANK_ETIMEOUT (-5) /* a bounded device-side wait gave up */
#define FRANK_ENCCL (-6)    /* reserved for the expert-parallel layer */

/* Thread-local message describing the last failure on this thread. */
const char* frank_last_error(void);

/* ABI version of this library (major*100 + minor). */
int frank_abi_version(void);

/* Number of SMs of the current device (used to size persistent grids). */
int frank_num_sms(void);

/*
 * out = gate * silu(up), silu(u) = u / (1 + exp(-u)), n elements.
 * Replaces @activation_components.swiglu (swiglu.mlir:16-51; oracle
 * oracles/activation.py:11-21).  dtype FRANK_F32 or FRANK_BF16 (all three
 * buffers share it; bf16 computes in fp32).
 */
int frank_swiglu(int dtype, const void* gate, const void* up, void* out,
                 int64_t n, void* stream);

/*
 * Softmax over experts then descending top-k, starting from fp32 logits
 * [E, T] (moe_ffn_block.mlir:72-128, oracles/moe.py:90-105).
 * Ties go to the lowest expert index.  Writes weights [k, T] fp32 and
 * ids [k, T] int32.  Exported so routing can be tested bit-exactly on
 * identical logits.
 */
int frank_softmax_topk(const float* logits, int64_t T, int64_t E, int64_t k,
                       int normalize, float* weights, int32_t* ids,
                       void* stream);

/*
 * Router: logits = wr @ x.T in fp32, then frank_softmax_topk's rule
 * (moe_ffn_block.mlir:54-128, oracles/moe.py:87-105).
 * x_dtype / wr_dtype: FRANK_F32 or FRANK_BF16.  E <= 256, 1 <= k <= min(E, 32).
 * logits_scratch: device scratch of frank_router_scratch_bytes(x_dtype, T,
 * H, E) bytes (0 when E <= 8), 256-byte aligned; with NULL a slower kernel
 * that needs no scratch is used.  With bf16 x, E a multiple of 16 and
 * T >= 128 the logits come from a tensor-core GEMM against wr split exactly
 * into three bf16 terms (hi + mid + lo), accumulated in fp32.
 */
size_t frank_router_scratch_bytes(int x_dtype, int64_t T, int64_t H,
                                  int64_t E);

/*
 * Router weights prepared once per block: an fp32 copy of wr [E, H]
 * followed (at byte offset frank_router_pack_offset(E, H)) by its exact
 * three-term bf16 split [3, E, H] (hi, mid = bf16(wr - hi),
 * lo = bf16(wr - hi - mid)).  Passing the pack with wr_dtype =
 * FRANK_ROUTER_PACKED to frank_router_topk, frank_moe_ffn_block or
 * frank_moe_ffn_sublayer gives the same results as passing wr itself; the
 * tensor-core router then skips rebuilding the split on every call.  No
 * counterpart in the reference (whose router is one fp32 matmul,
 * moe_ffn_block.mlir:54-70).  wr_dtype FRANK_F32 or FRANK_BF16; pack:
 * frank_router_pack_size(E, H) bytes, 256-byte aligned.
 */
size_t frank_router_pack_size(int64_t E, int64_t H);
size_t frank_router_pack_offset(int64_t E, int64_t H);
int frank_router_pack(int wr_dtype, const void* wr, int64_t E, int64_t H,
                      void* pack, void* stream);
int frank_router_topk(int x_dtype, const void* x, int wr_dtype, const void* wr,
                      int64_t T, int64_t H, int64_t E, int64_t k, int normalize,
                      float* weights, int32_t* ids, float* logits_scratch,
                      void* stream);

/*
 * Atomic-free, stable expert permutation of the flattened slots
 * s = j*T + t (slot-major, mul_mat_id.mlir:51-53).  Equivalent to
 * argsort(ids.reshape(-1), stable) and a bincount prefix:
 *   sorted_slots[k*T]  flat slot at each expert-sorted row
 *   offsets[E+1]       first sorted row of each expert
 *   slot_pos[k*T]      sorted row of each flat slot
 * workspace: frank_permute_workspace_size(k*T, E) bytes.  err_flag (device
 * int32, may be NULL) receives 1 when an id is outside [0, E); such ids are
 * clamped so that the call stays memory-safe.
 */
size_t frank_permute_workspace_size(int64_t n_slots, int64_t E);
int frank_permute(const int32_t* ids, int64_t n_slots, int64_t E,
                  int32_t* sorted_slots, int32_t* offsets, int32_t* slot_pos,
                  int32_t* err_flag, void* workspace, size_t ws_bytes,
                  void* stream);

/*
 * frank_permute without a workspace argument, for callers that cannot
 * allocate device memory (a host framework that owns the device memory
 * pool, an FFI binding that cannot keep a CUDA workspace alive, or a loop
 * where allocating is not allowed).  No counterpart in the reference: it is
 * an addition of this library.  Same inputs, outputs and results as
 * frank_permute; the scratch is a fixed library-owned device array of
 * FRANK_PERMUTE_NOALLOC_SCRATCH_BYTES, held by every GPU that loads the
 * library until exit.  Returns FRANK_EINVAL when
 * frank_permute_workspace_size(n_slots, E) exceeds it (1 MiB covers, e.g.,
 * 65536 slots with any E <= 1024).  The first call on a device looks up the
 * array's device address and should come before any stream capture; the
 * address is cached for the process's life (one context per device: do not
 * call it again after cudaDeviceReset).  All calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  Allocates nothing.
 */
#define FRANK_PERMUTE_NOALLOC_SCRATCH_BYTES (1u << 20)
int frank_permute_noalloc(const int32_t* ids, int64_t n_slots, int64_t E,
                          int32_t* sorted_slots, int32_t* offsets,
                          int32_t* slot_pos, int32_t* err_flag, void* stream);

/*
 * One-time weight prepack: [O, I, E] (expert innermost, in_dtype) ->
 * [E, O, I] (out_dtype).  Replaces the per-call transpose of
 * mul_mat_id.mlir:38-48.  FRANK_F32 -> FRANK_F32 or FRANK_BF16;
 * FRANK_BF16 -> FRANK_BF16.
 */
int frank_prepack_experts(int in_dtype, const void* w_oie, int64_t O,
                          int64_t I, int64_t E, int out_dtype, void* w_eoi,
                          void* stream);

/*
 * Expert-selected matmul, @moe_components.mul_mat_id (mul_mat_id.mlir:22-120,
 * oracles/moe.py:9-48):  out[:, j, t] = W[:, :, ids[j, t]] @ in[:, j, t].
 *   dtype FRANK_F32: w_eoi fp32 [E,O,I], input fp32 [I,k,T]  (fp32 FFMA path)
 *   dtype FRANK_BF16: w_eoi bf16 [E,O,I], input bf16 [I,k,T] (tcgen05 path)
 * out is fp32 [O, k, T].  err_flag as in frank_permute (may be NULL).
 */
size_t frank_mul_mat_id_workspace_size(int dtype, int64_t O, int64_t I,
                                       int64_t E, int64_t k, int64_t T);
int frank_mul_mat_id(int dtype, const void* w_eoi, const void* input,
                     const int32_t* ids, int64_t O, int64_t I, int64_t E,
                     int64_t k, int64_t T, float* out, int32_t* err_flag,
                     void* workspace, size_t ws_bytes, void* stream);

/*
 * Full MoE FFN block, @moe_ffn_components.moe_ffn_block
 * (moe_ffn_block.mlir:34-209, oracles/moe.py:51-132):
 *   route -> permute -> h = gate(x) * silu(up(x)) -> d = down(h) * w
 *   -> y[t] = sum_j d[slot j of t]  (j = 0..k-1 in order).
 *   dtype FRANK_F32 : x fp32 [T,H], packed weights fp32 (FFMA path)
 *   dtype FRANK_BF16: x bf16 [T,H], packed weights bf16 (tcgen05 path,
 *                     fp32 accumulation, h = swiglu(..) held in bf16)
 * y [T,H] has y_dtype: FRANK_F32 (the reference's output type,
 * moe_ffn_block.mlir:45) or FRANK_BF16.
 * wr [E, H] is fp32 or bf16 (wr_dtype).  Packed weights:
 *   w_up_p, w_gate_p [E, F, H]; w_down_p [E, H, F]  (frank_prepack_experts)
 * wr may also be a router pack (wr_dtype FRANK_ROUTER_PACKED).
 * Optional outputs (may be NULL): route_w [k,T] fp32, route_ids [k,T] int32.
 * Workspace header: the first FRANK_WORKSPACE_HEADER_BYTES of the workspace
 * hold the decode kernel's grid-barrier counters.  Zero them once before
 * the first call with a workspace (cudaMemset); every call leaves them zero
 * again (also one that gave up with FRANK_ETIMEOUT), so a workspace can be
 * reused, resized from the same base or captured in a CUDA graph without a
 * per-call reset.  Calls that share a workspace must not overlap.
 */
#define FRANK_WORKSPACE_HEADER_BYTES 256
size_t frank_moe_ffn_block_workspace_size(int dtype, int64_t T, int64_t H,
                                          int64_t F, int64_t E, int64_t k);
int frank_moe_ffn_block(int dtype, const void* x, int wr_dtype, const void* wr,
                        const void* w_up_p, const void* w_gate_p,
                        const void* w_down_p, int64_t T, int64_t E, int64_t k,
                        int64_t H, int64_t F, int normalize, int y_dtype, void* y,
                        float* route_w, int32_t* route_ids, void* workspace,
                        size_t ws_bytes, void* stream);

/*
 * rms_norm: out[t] = (x[t] / sqrt(mean(x[t]^2) + eps)) * weight, x [T, H]
 * fp32, weight [H] fp32, out [T, H] in out_dtype (FRANK_F32 or FRANK_BF16).
 * Replaces @rms_norm_components.rms_norm_linalg
 * (components/normalization/rms_norm.mlir:18-80; oracle
 * oracles/normalization.py:10-43).
 */
int frank_rms_norm(const float* x, const float* weight, int64_t T, int64_t H,
                   float eps, int out_dtype, void* out, void* stream);

/*
 * The MoE FFN sub-layer of the reference's MoE transformer layer
 * (architectures/llm/transformer_layer_moe_prefill.mlir:211-245 and the
 * decode layer's :228-256; oracle oracles/transformer_layer.py:107-124):
 *   out = residual + moe_ffn_block(rms_norm(residual, norm_w, eps), ...)
 * residual, out: fp32 [T, H] (out may alias residual: in-place update);
 * norm_w: fp32 [H].  The normalised tokens are rounded to `dtype` (the block's
 * compute dtype) in the workspace; the residual add is fused into the block's
 * final sum over the k slots.  Other arguments as frank_moe_ffn_block.
 * Workspace: frank_moe_ffn_sublayer_workspace_size(dtype, T, H, F, E, k),
 * with the same zeroed header as frank_moe_ffn_block's.
 */
size_t frank_moe_ffn_sublayer_workspace_size(int dtype, int64_t T, int64_t H,
                                             int64_t F, int64_t E, int64_t k);
int frank_moe_ffn_sublayer(int dtype, const float* residual,
                           const float* norm_w, float eps, int wr_dtype,
                           const void* wr, const void* w_up_p,
                           const void* w_gate_p, const void* w_down_p,
                           int64_t T, int64_t E, int64_t k, int64_t H,
                           int64_t F, int normalize, float* out,
                           float* route_w, int32_t* route_ids, void* workspace,
                           size_t ws_bytes, void* stream);

/*
 * Building blocks of moe_ffn_block, exported for the expert-parallel layer
 * (which runs the stages with NCCL exchanges in between):
 *
 * frank_gather_rows: xs[r, :] = x[sorted_slots[r] % T, :] (the replicate +
 *   permute of moe_ffn_block.mlir:130-144 / mul_mat_id.mlir:64-84).
 * frank_gather_weights: w_sorted[r] = w[sorted_slots[r]].
 * frank_expert_ffn: for expert-sorted rows xs [rows, H] with expert row
 *   offsets [E+1] and per-row gate weights: d = (gate(xs) * silu(up(xs)))
 *   @ down^T * w_rows, fp32 [rows, H] (moe_ffn_block.mlir:146-177).
 *   Workspace: frank_expert_ffn_workspace_size(dtype, rows, F).
 * frank_combine: y[t] = sum_{j<k} d[slot_pos[j*T + t]] in order j
 *   (moe_ffn_block.mlir:179-206); y_dtype FRANK_F32 or FRANK_BF16.
 * frank_copy_row_segments: dst rows [dst_start[s], +len) = src rows
 *   [src_start[s], +len) for nseg segments; seg_prefix [nseg+1] is the
 *   exclusive prefix of the lengths (device int64 arrays); row_bytes % 4 == 0.
 */
int frank_gather_rows(int dtype, const void* x, const int32_t* sorted_slots,
                      int64_t rows, int64_t T, int64_t H, void* xs,
                      void* stream);
int frank_gather_weights(const float* w, const int32_t* sorted_slots,
                         int64_t n, float* w_sorted, void* stream);
size_t frank_expert_ffn_workspace_size(int dtype, int64_t rows, int64_t F);
int frank_expert_ffn(int dtype, const void* xs, const float* w_rows,
                     const int32_t* offsets, int64_t E, int64_t rows,
                     int64_t H, int64_t F, const void* w_up_p,
                     const void* w_gate_p, const void* w_down_p, float* d,
                     void* workspace, size_t ws_bytes, void* stream);
int frank_combine(const float* d, const int32_t* slot_pos, int64_t T,
                  int64_t k, int64_t H, int y_dtype, void* y, void* stream);
int frank_copy_row_segments(const void* src, void* dst,
                            const int64_t* src_start, const int64_t* dst_start,
                            const int64_t* seg_prefix, int64_t nseg,
                            int64_t total_rows, int64_t row_bytes,
                            void* stream);

/*
 * Expert-parallel exchange over NVLink peer memory (no counterpart in the
 * reference, which runs on one device).  E experts are split evenly over P
 * ranks (El = E / P each, contiguous).  counts_all [P][E] int32 holds every
 * rank's per-expert row counts (all-gathered by the caller).
 *
 * frank_ep_plan: dst_base [E] = first row of this rank's chunk for expert g
 *   in the owning rank's expert-major receive buffer; local_offsets [El+1] =
 *   this rank's expert row offsets; row_rank / row_pos [capacity] = for each
 *   received row, the source rank and its row in that rank's expert-sorted
 *   order (filled for the rows actually received, below `capacity`).
 * frank_ep_dispatch: for this rank's n_slots expert-sorted slots, copies the
 *   bf16 token row x[sorted_slots[r] % T] and gate weight w[sorted_slots[r]]
 *   into peer_x[p] / peer_w[p] (device addresses of every rank's receive
 *   buffers of `capacity` rows, P <= 8) at the planned rows.  A planned row
 *   outside [0, capacity) is skipped and FRANK_EINVAL is recorded in
 *   *overflow, or in the device error word (frank_read_device_error) when
 *   overflow is NULL.  A caller that plans with receive buffers sized from
 *   an earlier step and checks this step's counts on the host afterwards
 *   (redoing the step when they did not fit) passes its own overflow word.
 * frank_expert_ffn_scatter: frank_expert_ffn (bf16) whose fp32 output row r
 *   is stored at peer_out[row_rank[r]] + row_pos[r] * H, i.e. straight into
 *   the return buffer of the rank the row came from.  Every return buffer
 *   holds peer_rows rows; a map entry outside [0, n_peers) x [0, peer_rows)
 *   is not stored and records FRANK_EINVAL in the device error word.
 * frank_ep_plan clamps the local expert offsets to `capacity`, so rows
 *   beyond the receive buffer are never read by the GEMMs either (and
 *   FRANK_EINVAL is recorded, in *overflow if given, when the gathered
 *   counts exceed it).
 * Stores to other GPUs complete with the kernels; the caller orders the
 *   ranks' steps (e.g. an NCCL collective on the same stream) before a rank
 *   reads what its peers wrote.  No kernel here waits on another GPU.
 */
int frank_ep_plan(const int32_t* counts_all, int P, int El, int rank,
                  int32_t* dst_base, int32_t* local_offsets, int32_t* row_rank,
                  int32_t* row_pos, int64_t capacity, int32_t* overflow,
                  void* stream);
int frank_ep_dispatch(const void* x, int64_t T, int64_t H, const float* w,
                      const int32_t* sorted_slots, const int32_t* offsets,
                      int64_t E, int64_t El, int64_t n_slots,
                      const int32_t* dst_base, void* const* peer_x,
                      float* const* peer_w, int P, int64_t capacity,
                      int32_t* overflow, void* stream);
int frank_expert_ffn_scatter(const void* xs, const float* w_rows,
                             const int32_t* offsets, int64_t E, int64_t rows,
                             int64_t H, int64_t F, const void* w_up_p,
                             const void* w_gate_p, const void* w_down_p,
                             const int32_t* row_rank, const int32_t* row_pos,
                             void* const* peer_out, int n_peers,
                             int64_t peer_rows, void* workspace,
                             size_t ws_bytes, void* stream);

/*
 * Device error word written by bounded waits inside the persistent GEMM
 * kernels (0 = none).  frank_read_device_error copies it to *out and resets
 * it; synchronises the stream.
 */
int frank_read_device_error(int32_t* out, void* stream);

/*
 * Failure-detection self-test (no counterpart in the reference): runs the
 * library's bounded mbarrier wait on a barrier that nothing completes, with
 * the given limit in nanoseconds.  The wait must give up: *completed
 * receives 0 and the device error word holds FRANK_ETIMEOUT (read and clear
 * it with frank_read_device_error).  Synchronises the stream.
 */
int frank_selftest_bounded_wait(int64_t limit_ns, int32_t* completed,
                                void* stream);

/* Number of kernels this library has launched in this process. */
uint64_t frank_launch_count(void);

/*
 * Stage timing for measurement tools.  While enabled, frank_moe_ffn_block
 * records a CUDA event on the caller's stream before its first stage and
 * after each stage:  0 route (router + softmax + top-k), 1 permute,
 * 2 gather of expert-sorted rows, 3 gate/up GEMM + swiglu, 4 down GEMM,
 * 5 combine.  Up to 64 calls are recorded per window.  frank_profile_read
 * waits for the last recorded call, writes up to max_stages mean durations
 * in milliseconds over the window's calls, stores the number of calls in
 * *n_stages and starts a new window.  Events belong to the device current at
 * the first enabled call.  Measurement only; off by default.
 * enable = 2 is the graph-capture form: every call records into the same
 * single event set (so a captured graph re-records it on each replay) and
 * reading does not clear it.
 */
int frank_profile_stages(int enable);
int frank_profile_read(float* stage_ms, int max_stages, int* n_stages);

#ifdef __cplusplus
}
#endif

#endif /* FRANK_MOE_H_ */
