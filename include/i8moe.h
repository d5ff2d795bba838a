/*
 * i8moe.h -- C ABI of libi8moe.so, the sm_100a (B200) implementation of the
 * INT8 hybrid MoE forward path of PatchouliTIS/INT8BlockwiseGEMM.
 *
 * Conventions
 *  - Every pointer is a device pointer unless stated otherwise; every tensor
 *    is dense and row-major.  The caller allocates every output (the
 *    reference ops are all out-parameter style).
 *  - Every entry point launches asynchronously on `stream` (a cudaStream_t)
 *    on the current device and never synchronises.
 *  - Return value: I8MOE_OK (0) or a negative I8MOE_ERR_* code;
 *    i8moe_last_error() then returns a message (per calling thread).
 *  - Kernels never trap.  A device-side wait that times out or an index that
 *    fails a bounds check sets a bit in a per-device error word that
 *    i8moe_device_error() reads.
 *  - Reference locations are given as path:line inside the reference
 *    project.
 */
#ifndef I8MOE_H_
#define I8MOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* i8moe_stream_t; /* cudaStream_t */

enum {
  I8MOE_OK = 0,
  I8MOE_ERR_INVALID = -1,     /* bad argument (the reference's TORCH_CHECK cases) */
  I8MOE_ERR_CUDA = -2,        /* a CUDA runtime / driver call failed */
  I8MOE_ERR_UNSUPPORTED = -3, /* device is not sm_100 or shape outside supported range */
};

/* Element types of activations / outputs.  I8MOE_S32 is accepted only as a
 * GEMM output: it stores the raw int32 accumulator W (before the float
 * epilogue) for bit-exact verification. */
enum { I8MOE_BF16 = 0, I8MOE_FP16 = 1, I8MOE_FP32 = 2, I8MOE_S32 = 3 };

/* ---------------------------------------------------------------- misc */

int i8moe_abi_version(void);
const char* i8moe_last_error(void);
/* Reads (and with clear != 0 resets) the device error word of `device`. */
int i8moe_device_error(int device, uint32_t* word, int clear);
/* Replaces moe_permute_unpermute_supported
 * (csrc/moe_permute_unpermute_op.cu:258-264, schema csrc/torch_bindings.cpp:127):
 * 1, because the library is built with CUDA >= 12 (no device needed). */
int i8moe_moe_permute_unpermute_supported(void);

/* ------------------------------------------------------------- routing */

/* Bytes of scratch the routing entry points need for n_rows = n_token*topk
 * keys of n_expert experts. */
size_t i8moe_route_workspace_size(int64_t n_rows, int64_t n_expert);

/* Replaces moe_permute_metadata (csrc/moe_permute_unpermute_op.cu:81-132,
 * schema csrc/torch_bindings.cpp:116-120).  Stable sort of the expanded rows
 * by expert id:
 *   expert_first_token_offset[n_local_expert+1] (int64),
 *   inv_permuted_idx[n_token*topk]  (source expanded row -> destination),
 *   permuted_idx[n_token*topk]      (destination -> source; slots past
 *       expert_first_token_offset[n_local_expert] -- rows of no local
 *       expert, when expert_map != NULL -- get the sentinel n_token*topk,
 *       the value the reference pre-fills them with).
 * token_expert_indices supplies the value sorted with each key (the
 * reference passes arange; NULL means arange).  expert_map (nullable,
 * [n_expert]) remaps
 * global ids for expert parallelism as the reference does.  `workspace` must
 * hold i8moe_route_workspace_size() bytes. */
int i8moe_moe_permute_metadata(const int32_t* topk_ids, const int32_t* token_expert_indices,
                               const int32_t* expert_map, int64_t n_token, int64_t topk,
                               int64_t n_expert, int64_t n_local_expert,
                               int64_t* expert_first_token_offset, int32_t* inv_permuted_idx,
                               int32_t* permuted_idx, void* workspace, size_t workspace_bytes,
                               i8moe_stream_t stream);

/* No reference counterpart.  moe_permute_metadata for callers that cannot
 * allocate device memory per call: identical arguments and results to
 * i8moe_moe_permute_metadata minus the workspace, whose role is taken by a
 * fixed 1 MiB device array inside the library (so it needs
 * i8moe_route_workspace_size(n_token*topk, n_expert) <= 1048576 bytes, e.g.
 * up to 1,048,576 rows at 256 experts; larger problems return
 * I8MOE_ERR_INVALID and must use the workspace entry point).  The first call
 * on a device looks the array up with cudaGetSymbolAddress, so make it before
 * any stream capture on that device.  The array is shared by every call on a
 * device: calls that overlap on one device race and must be serialised by the
 * caller.  Nothing is allocated. */
int i8moe_moe_permute_metadata_noalloc(const int32_t* topk_ids,
                                       const int32_t* token_expert_indices,
                                       const int32_t* expert_map, int64_t n_token, int64_t topk,
                                       int64_t n_expert, int64_t n_local_expert,
                                       int64_t* expert_first_token_offset,
                                       int32_t* inv_permuted_idx, int32_t* permuted_idx,
                                       i8moe_stream_t stream);

/* No reference counterpart (the router runs before the reference's runner,
 * which takes topk_ids / topk_weights).  Per token: the top-k experts by
 * logits + bias (ties to the lower id) and, as their weights, the softmax of
 * their unbiased logits (renormalised over the top-k).  logits [T, E] fp32,
 * bias [E] fp32 or NULL, E <= 1024, topk <= min(32, E); topk_ids [T, k]
 * int32, topk_weights [T, k] fp32. */
int i8moe_router_topk(const float* logits, const float* bias, int64_t n_token, int64_t n_expert,
                      int64_t topk, int32_t* topk_ids, float* topk_weights,
                      i8moe_stream_t stream);

/* No reference counterpart: i8moe_router_topk fused with the routing of
 * i8moe_moe_route_for_gemm -- the router kernel writes topk_ids / weights and
 * the routing histogram in one pass, then the offsets, problem sizes, scale
 * offsets and permutation maps follow as in i8moe_moe_route_for_gemm (same
 * arguments after topk_weights, same workspace). */
int i8moe_router_route_for_gemm(const float* logits, const float* bias, int64_t n_token,
                                int64_t n_expert, int64_t topk, int32_t* topk_ids,
                                float* topk_weights, const int32_t* token_expert_indices,
                                const int32_t* expert_map, int64_t n_local_expert,
                                int64_t* expert_first_token_offset, int32_t* inv_permuted_idx,
                                int32_t* permuted_idx, int32_t* expert_offsets,
                                int32_t* problem_sizes13, int32_t* problem_sizes2,
                                int32_t* scale_offsets, int64_t n_out1, int64_t k1,
                                int64_t n_out2, int64_t k2, int64_t tile_m, void* workspace,
                                size_t workspace_bytes, i8moe_stream_t stream);

/* Fused-forward variant of i8moe_moe_permute_metadata (no reference
 * counterpart; it replaces the host-side torch glue of the reference runner,
 * int8_hybrid_moe/cutlass_runner.py:136-143 and the scale-offset cumsum of
 * int8_hybrid_moe/quant.py:391-395).  Besides the routing maps it writes
 *   expert_offsets [n_local+1] int32, problem_sizes13 / problem_sizes2
 *   [n_local, 3] int32 = (M_e, n_out1, k1) / (M_e, n_out2, k2), and
 *   scale_offsets [n_local+1] int32 = exclusive cumsum of ceil(M_e/tile_m),
 * from the same kernels, so the forward needs no extra launches. */
int i8moe_moe_route_for_gemm(const int32_t* topk_ids, const int32_t* token_expert_indices,
                             const int32_t* expert_map, int64_t n_token, int64_t topk,
                             int64_t n_expert, int64_t n_local_expert,
                             int64_t* expert_first_token_offset, int32_t* inv_permuted_idx,
                             int32_t* permuted_idx, int32_t* expert_offsets,
                             int32_t* problem_sizes13, int32_t* problem_sizes2,
                             int32_t* scale_offsets, int64_t n_out1, int64_t k1, int64_t n_out2,
                             int64_t k2, int64_t tile_m, void* workspace,
                             size_t workspace_bytes, i8moe_stream_t stream);

/* Replaces moe_permute (csrc/moe_permute_unpermute_op.cu:10-79, schema
 * csrc/torch_bindings.cpp:109-114): the metadata above plus the row gather
 * permuted_input[d] = input[permuted_idx[d] / topk] (expandInputRowsKernel,
 * permute_unpermute_kernels/moe_permute_unpermute_kernel.inl:3-78). */
int i8moe_moe_permute(const void* input, int dtype, int64_t n_hidden, const int32_t* topk_ids,
                      const int32_t* token_expert_indices, const int32_t* expert_map,
                      int64_t n_token, int64_t topk, int64_t n_expert, int64_t n_local_expert,
                      void* permuted_input, int64_t* expert_first_token_offset,
                      int32_t* inv_permuted_idx, int32_t* permuted_idx, void* workspace,
                      size_t workspace_bytes, i8moe_stream_t stream);

/* Replaces moe_unpermute (csrc/moe_permute_unpermute_op.cu:134-169,
 * finalizeMoeRoutingKernel moe_permute_unpermute_kernel.inl:132-206):
 *   out[t] = dtype( sum_j fma(topk_weights[t,j], permuted[inv[t,j]], acc) )
 * skipping rows >= expert_first_token_offset[n_local_expert] when that
 * pointer is non-NULL. */
int i8moe_moe_unpermute(const void* permuted_hidden, int dtype, const float* topk_weights,
                        const int32_t* inv_permuted_idx,
                        const int64_t* expert_first_token_offset, int64_t n_local_expert,
                        int64_t n_token, int64_t topk, int64_t n_hidden, void* out,
                        i8moe_stream_t stream);

/* ---------------------------------------------------------- activation */

/* Replaces silu_and_mul (csrc/activation_kernels.cu:260-265):
 * out[r, i] = dtype(silu(x[r, i])) * x[r, d + i], x is [n_rows, 2d]. */
int i8moe_silu_and_mul(void* out, const void* input, int dtype, int64_t n_rows, int64_t d,
                       i8moe_stream_t stream);

/* ---------------------------------------------------------------- quant */

/* Scale rows of one grouped quant: scale_offsets[E+1] = exclusive cumsum of
 * ceil((expert_offsets[e+1]-expert_offsets[e]) / tile_m)
 * (int8_hybrid_moe/quant.py:238-242). */
int i8moe_scale_offsets(const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int32_t* scale_offsets, i8moe_stream_t stream);

/* Per-(expert M-tile x 128-K block) absmax INT8 quantisation with the
 * two-level (Q int32, F fp32) scale factorisation folded in.
 *
 * Replaces, for the three activation sources:
 *   i8moe_quant_grouped  -- moe_kernel_quantize_input_int8_hybrid_grouped
 *                           (int8_hybrid_moe/quant.py:147-277), A is [M, K]
 *   i8moe_quant_permute  -- fused_permute_quant_int8_hybrid_grouped
 *                           (quant.py:284-433), rows hidden[permuted_idx/topk]
 *   i8moe_quant_silu     -- fused_silu_quant_int8_hybrid_grouped
 *                           (quant.py:440-579), x = silu(gate) * up of mm1
 *                           [M, 2K]
 * followed by quantize_scales_for_hybrid (quant.py:52-140).
 * Outputs: qA [M, K] int8 (rows outside every expert untouched),
 *          Q [rows_upper, Kb] int32, F [rows_upper, ceil(Kb/super_group)],
 *          where only the first scale_offsets[E] rows are written;
 *          scale_offsets [E+1] int32 (computed here when
 *          `scale_offsets_ready` == 0, read as given otherwise).
 * block_k must be 128; K % 8 == 0. */
int i8moe_quant_grouped(const void* A, int dtype, int64_t M, int64_t K,
                        const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                        int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                        i8moe_stream_t stream);
int i8moe_quant_permute(const void* hidden, int dtype, int64_t n_token, int64_t K,
                        const int32_t* permuted_idx, int64_t M, int64_t topk,
                        const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                        int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                        int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                        i8moe_stream_t stream);
int i8moe_quant_silu(const void* mm1, int dtype, int64_t M, int64_t N,
                     const int32_t* expert_offsets, int64_t n_expert, int64_t tile_m,
                     int64_t block_k, int64_t q_max, int64_t super_group_size, int8_t* qA,
                     int32_t* Q, float* F, int32_t* scale_offsets, int scale_offsets_ready,
                     i8moe_stream_t stream);

/* Replaces the reference's weight preparation _quantize_blockwise_int8
 * (bench_int8_hybrid_moe.py:98-120, called with block_n = 64, block_k =
 * quant_block_size at :220-229), which is host-side torch code there.  Per
 * (expert, 64-row, 128-column) block of w [E, N, K] (bf16 / fp16 / fp32):
 * scale = max(absmax, 1e-10) / 127 and q = clamp(rint(w / scale), -128, 127)
 * (ties to even), ragged blocks padded with zeros.  q [E, N, K] int8, scale
 * [E, ceil(N/64), ceil(K/128)] fp32.  The GEMM's Q_B / F_B follow with
 * i8moe_quantize_scales over the [E * ceil(N/64), ceil(K/128)] view. */
int i8moe_quantize_weights(const void* w, int dtype, int64_t n_expert, int64_t n, int64_t k,
                           int64_t block_n, int64_t block_k, int8_t* q, float* scale,
                           i8moe_stream_t stream);

/* Replaces quantize_scales_for_hybrid (int8_hybrid_moe/quant.py:52-140) on a
 * standalone fp32 scale matrix [rows, kb]. */
int i8moe_quantize_scales(const float* scale, int64_t rows, int64_t kb, int64_t q_max,
                          int64_t super_group_size, int32_t* Q, float* F,
                          i8moe_stream_t stream);

/* ---------------------------------------------------------------- GEMMs */

/* Replaces cutlass_int8_blockwise_hybrid_grouped{,_small}{,_bias}
 * (csrc/int8_hybrid_grouped_gemm.cu:757-805, schemas
 * csrc/torch_bindings.cpp:80-106).  tcgen05 kind::i8 persistent grouped GEMM:
 *   W[r,n]   = sum_qb (a_qscale[s,qb] * b_qscale[e,n/64,qb]) *
 *              sum_{k in qb} a_q[r,k] * b_q[e,n,k]        (int32, wrapping)
 *   out[r,n] = out_dtype( float(W) * (a_fscale[s,0] * b_fscale[e,n/64,0]) [+ bias] )
 * with s = scale_offsets[e] + (r - expert_offsets[e]) / tile_m
 * (tile_m 128 = default variant, 64 = _small variant).  a_q [sum_m, k],
 * b_q [n_expert, n, k], out [sum_m, n]; problem_sizes [n_expert, 3]
 * (M_e, n, k).  scale_offsets may be NULL (then derived from
 * problem_sizes); bias NULL or fp32 [n] (bias_stride 0) / [n_expert, n]
 * (bias_stride n).  out_dtype I8MOE_BF16 (the reference's only output),
 * I8MOE_FP16, or I8MOE_S32 (raw W, no bias).  Requires k % 32 == 0, n % 8 == 0,
 * quant_block_size % 128 == 0. */
int i8moe_hybrid_grouped_gemm(const int8_t* a_q, const int32_t* a_qscale, const float* a_fscale,
                              int64_t a_scale_rows, const int8_t* b_q, const int32_t* b_qscale,
                              const float* b_fscale, const int32_t* expert_offsets,
                              const int32_t* problem_sizes, const int32_t* scale_offsets,
                              const float* bias, int64_t bias_stride, void* out, int out_dtype,
                              int64_t n_expert, int64_t sum_m, int64_t n, int64_t k,
                              int64_t quant_block_size, int64_t super_group_size,
                              int64_t tile_m, i8moe_stream_t stream);

/* No reference counterpart: the w13 hybrid GEMM with the SiLU*up + INT8
 * requant of the intermediate fused into its epilogue.  It produces exactly
 * what i8moe_hybrid_grouped_gemm (w13, out_dtype = act_dtype) followed by
 * i8moe_quant_silu would (reference int8_hybrid_grouped_gemm.cu:218-479 then
 * quant.py:440-579), without writing the [sum_m, 2N] intermediate.
 *   w13_q [E, 2N, K] int8 (gate rows 0..N-1, up rows N..2N-1) with its Q/F,
 *   act_dtype   storage type of the intermediate (I8MOE_BF16 / I8MOE_FP16),
 *   n_act = N   (a multiple of 32),
 *   scale_offsets [E+1] int32 (entry E = total scale rows), as written by
 *               i8moe_moe_route_for_gemm / i8moe_scale_offsets for tile_m,
 *   act_q [sum_m, N] int8, act_qscale [ceil(sum_m/tile_m)+E, ceil(N/128)]
 *   int32, act_fscale [same rows, ceil(ceil(N/128)/super_group_size)] fp32. */
int i8moe_hybrid_grouped_gemm_silu_quant(
    const int8_t* a_q, const int32_t* a_qscale, const float* a_fscale, int64_t a_scale_rows,
    const int8_t* w13_q, const int32_t* w13_qscale, const float* w13_fscale,
    const int32_t* expert_offsets, const int32_t* problem_sizes, const int32_t* scale_offsets,
    const float* bias, int64_t bias_stride, int act_dtype, int64_t n_expert, int64_t sum_m,
    int64_t n_act, int64_t k, int64_t quant_block_size, int64_t super_group_size,
    int64_t tile_m, int64_t q_max, int8_t* act_q, int32_t* act_qscale, float* act_fscale,
    i8moe_stream_t stream);

/* Replaces cutlass_int8_grouped_mm (csrc/int8_grouped_gemm.cu:106-220,
 * schema csrc/torch_bindings.cpp:75-78):
 *   out[r,n] = out_dtype(float(sum_k a[r,k]*b[e,n,k]) * alpha_r)
 * alpha_r = alpha (per tensor; the reference's float(a_scale*b_scale)), or,
 * when a_row_scale and b_expert_scale are both non-NULL,
 * alpha_r = a_row_scale[r] * b_expert_scale[e] (per-token x per-expert
 * extension).  No host synchronisation. */
int i8moe_int8_grouped_mm(const int8_t* a, const int8_t* b, void* out, int out_dtype,
                          float alpha, const float* a_row_scale, const float* b_expert_scale,
                          const int32_t* expert_offsets, const int32_t* problem_sizes,
                          int64_t n_expert, int64_t sum_m, int64_t n, int64_t k,
                          i8moe_stream_t stream);

/* Grouped-GEMM variant (no reference counterpart; results are identical
 * either way).  mode 1: every hybrid grouped GEMM above runs on CTA pairs --
 * clusters of two CTAs sharing one tcgen05.mma.cta_group::2 over 256-row
 * pair tiles of one expert, each CTA streaming half of the weight tile;
 * mode 0 and mode -1 (default): one CTA per 128-row tile (measured faster
 * at the benchmark shapes).  Process-wide; returns the previous mode, or
 * I8MOE_ERR_INVALID for another value. */
int i8moe_gemm_set_cta_pairs(int mode);

/* No reference counterpart: the measured dense INT8 tensor-core peak.
 * Launches one CTA per SM (cta_group 1) or one CTA pair per two SMs
 * (cta_group 2, M = 256), each issuing `steps` x 4 tcgen05.mma kind::i8
 * (M x 256 x 32) back to back from shared memory into TMEM, nothing else.
 * The caller times the launch on `stream`; each CTA performs
 * 2 * 128 * 256 * 128 * steps int8 operations, and *n_cta receives the
 * number of CTAs launched.  The denominator of the INT8 roofline fractions. */
int i8moe_int8_mma_peak(int64_t steps, int cta_group, int64_t* n_cta, i8moe_stream_t stream);

/* ---------------------------------------------------- expert parallelism */
/* No reference counterpart: the device-side bookkeeping of the expert-
 * parallel dispatch and combine (the all-to-alls themselves are NCCL calls
 * made by the host).  Rank d owns experts [d*n_local, (d+1)*n_local).
 *
 * ep_plan: for every token t and rank d, pos[t, d] = slot of t in d's send
 *   segment (tokens in order) or -1; token_list [n_rank, n_token] holds each
 *   segment's tokens; counts [n_rank] int32 the segment lengths. */
int i8moe_ep_plan(const int32_t* topk_ids, int64_t n_token, int64_t topk, int64_t n_local_expert,
                  int64_t n_rank, int32_t* pos, int32_t* token_list, int32_t* counts,
                  i8moe_stream_t stream);
/* ep_pack: rows of `hidden` (row_bytes each, a multiple of 16) of every
 * segment, segment after segment, into send_rows; per row a meta row of its k
 * ids followed by the bits of its k weights into send_meta [rows, 2k] int32.
 * `counts` is a HOST array of the n_rank segment lengths. */
int i8moe_ep_pack(const void* hidden, int64_t row_bytes, const int32_t* topk_ids,
                  const float* topk_weights, int64_t topk, const int32_t* token_list,
                  int64_t n_token, int64_t n_rank, const int64_t* counts, void* send_rows,
                  int32_t* send_meta, i8moe_stream_t stream);
/* ep_combine: out[t] = dtype(sum over ranks d in order of back[off_d +
 * pos[t, d]]) with fp32 accumulation; back holds the returned partial rows
 * segment by segment (HOST `counts` as for ep_pack). */
int i8moe_ep_combine(const void* back, int dtype, const int32_t* pos, int64_t n_token,
                     int64_t n_rank, const int64_t* counts, int64_t n_hidden, void* out,
                     i8moe_stream_t stream);

/* ----------------------------------------- expert parallelism, peer memory */
/* No reference counterpart: the same dispatch / combine without NCCL and
 * without any host synchronisation, over NVLink peer memory.  Each rank
 * allocates one region (i8moe_ep_ipc_alloc), exchanges the 64-byte IPC
 * handles with the other ranks (any host channel) and maps theirs
 * (i8moe_ep_ipc_open).  A step on every rank, in order on one stream:
 *   i8moe_ep_plan          (pos, token_list, counts: device arrays)
 *   i8moe_ep_p2p_dispatch  rows, ids and weights into the destinations'
 *                          receive buffers; waits (bounded) for the peers'
 *                          segment lengths
 *   i8moe_ep_p2p_wait      until every source's rows have arrived
 *   the local forward over the `capacity` receive rows (rows past the
 *                          received ones carry `pad_expert`, an expert of
 *                          another rank, so the local routing skips them),
 *                          writing its [capacity, n_hidden] output into the
 *                          region's output buffer of the step's parity
 *   i8moe_ep_p2p_ready     announces that output to the peers
 *   i8moe_ep_p2p_combine   sums each token's partial rows from the peers'
 *                          output buffers in rank order (fp32) into out.
 * `par` is the step number modulo 2 (the same on every rank).  Waits give
 * up after 2 s and set a bit in i8moe_device_error.  No multicast objects
 * are created.
 *
 * Two combines, chosen when the region is sized (ROWS moves fewer NVLink
 * bytes; TOPK gives the single-GPU result bit for bit):
 *   I8MOE_EP_COMBINE_ROWS  the local forward ends with the top-k weighted
 *                          unpermute over this rank's experts (the
 *                          reference's expert_map skip,
 *                          moe_permute_unpermute_kernel.inl:133-190) into
 *                          the region's [capacity, n_hidden] output buffer;
 *                          i8moe_ep_p2p_combine adds the partial rows.
 *   I8MOE_EP_COMBINE_TOPK  the local forward stops after the w2 GEMM: its
 *                          mm2 rows [capacity * topk, n_hidden] and the
 *                          routing's inverse map [capacity, topk] go into
 *                          the region's mm2 / inv buffers, and
 *                          i8moe_ep_p2p_combine_topk performs the top-k
 *                          weighted unpermute itself, reading every slot's
 *                          mm2 row from the rank that owns its expert:
 *                          out[t] = dtype(sum over j in top-k order of
 *                          w[t, j] * mm2), one fp32 fma chain and one
 *                          rounding, as the single-GPU unpermute. */
#define I8MOE_IPC_HANDLE_BYTES 64
#define I8MOE_EP_COMBINE_ROWS 0
#define I8MOE_EP_COMBINE_TOPK 1

typedef struct {
  int64_t off_rows, off_ids, off_w, off_out, out_bytes, off_inbox, off_flags, off_epoch;
  int64_t off_mm2, mm2_bytes, off_inv, inv_bytes; /* per parity; 0 unless COMBINE_TOPK */
  int64_t bytes; /* region size */
} i8moe_ep_p2p_layout;

typedef struct {
  void* bases[32];        /* every rank's region, mapped in this process */
  int64_t n_rank, rank;
  int64_t n_token;        /* tokens of this rank */
  int64_t capacity;       /* receive rows: n_rank x max tokens per rank */
  int64_t topk, n_hidden, elem_bytes; /* elem_bytes: 2 (bf16 / fp16) */
  int64_t pad_expert;     /* a global expert id owned by another rank */
  i8moe_ep_p2p_layout layout;
} i8moe_ep_p2p;

/* combine: I8MOE_EP_COMBINE_ROWS or I8MOE_EP_COMBINE_TOPK */
int i8moe_ep_p2p_region_bytes(int64_t n_rank, int64_t capacity, int64_t topk, int64_t n_hidden,
                              int64_t elem_bytes, int combine, i8moe_ep_p2p_layout* layout);
/* cudaMalloc'd (zeroed) region and its IPC handle (I8MOE_IPC_HANDLE_BYTES) */
int i8moe_ep_ipc_alloc(int64_t bytes, void** ptr, uint8_t* handle);
int i8moe_ep_ipc_open(const uint8_t* handle, void** ptr);
int i8moe_ep_ipc_close(void* ptr);
int i8moe_ep_ipc_free(void* ptr);
int i8moe_ep_p2p_dispatch(const i8moe_ep_p2p* x, int par, const void* hidden,
                          const int32_t* topk_ids, const float* topk_weights,
                          const int32_t* token_list, const int32_t* counts,
                          i8moe_stream_t stream);
int i8moe_ep_p2p_wait(const i8moe_ep_p2p* x, int par, i8moe_stream_t stream);
int i8moe_ep_p2p_ready(const i8moe_ep_p2p* x, int par, i8moe_stream_t stream);
int i8moe_ep_p2p_combine(const i8moe_ep_p2p* x, int par, int dtype, const int32_t* pos, void* out,
                         i8moe_stream_t stream);
/* I8MOE_EP_COMBINE_TOPK: waits (bounded) for every destination's output,
 * then out[t] = dtype(sum_j w[t, j] * mm2_d[inv_d[row_d(t), j]]) in top-k
 * order with fp32 fmas, d = topk_ids[t, j] / n_local_expert and row_d(t)
 * the token's receive row at d (its segment offset + pos[t, d]). */
int i8moe_ep_p2p_combine_topk(const i8moe_ep_p2p* x, int par, int dtype, const int32_t* pos,
                              const int32_t* topk_ids, const float* topk_weights,
                              int64_t n_local_expert, void* out, i8moe_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* I8MOE_H_ */
