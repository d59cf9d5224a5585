/*
 * moe_b200.h — C ABI of the B200 (sm_100a) MoE operator library.
 *
 * Every entry point:
 *   - takes device pointers the caller allocated (outputs and workspace included);
 *   - enqueues its kernels on the given CUDA stream (`stream` is a cudaStream_t,
 *     NULL = legacy default stream) and never synchronises the host;
 *   - returns 0 on success or a positive MOE_ERR_* code; the message for the last
 *     failure on the calling thread is available from moe_last_error_string().
 * No C++ exceptions and no torch types cross this boundary.
 *
 * Tensor layouts are row-major and contiguous.  `dtype` codes: MOE_F32, MOE_F16, MOE_BF16.
 * Offsets follow the reference's grouped-GEMM contract: `num_offsets` is E+1
 * (offsets[0] = 0, offsets[e+1] = end row of expert e) or E (offsets[e] = end row).
 *
 * Each declaration cites the reference interface (echogujy/moe_ops, package
 * triton_gmm_ops) that it replaces.
 */
#ifndef MOE_B200_H_
#define MOE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum moe_dtype { MOE_F32 = 0, MOE_F16 = 1, MOE_BF16 = 2 };

enum moe_status {
  MOE_OK = 0,
  MOE_ERR_INVALID_ARG = 1,   /* bad shape / dtype / pointer combination          */
  MOE_ERR_UNSUPPORTED = 2,   /* valid request this build does not implement      */
  MOE_ERR_CUDA = 3,          /* a CUDA runtime call or kernel launch failed       */
  MOE_ERR_WORKSPACE = 4,     /* workspace missing or smaller than required        */
  MOE_ERR_DEVICE = 5         /* a kernel reported a device-side error flag        */
};

/* Library version string, e.g. "moe_b200 0.1.0 sm_100a". */
const char* moe_version(void);

/* Message describing the last non-zero status returned on this host thread. */
const char* moe_last_error_string(void);

/* Reads and clears the library's device-side error word on the current device
 * (synchronises the device).  0 = no error; 1 = a bounded wait inside a GEMM
 * kernel gave up; 2 = an expert index outside [0, E) was seen by permute. */
int moe_read_device_error(int* code_out);

/* Copies the device-side error word (4 bytes, not cleared) into `dst` (device or pinned host
 * memory) on `stream`, without synchronising: a caller can check it a step later. */
int moe_peek_device_error(void* dst, void* stream);

/* Failure-detection self-test (no counterpart in the reference): a kernel waits on an
 * mbarrier nothing arrives at, with the bounded wait every GEMM pipeline wait uses.  After
 * timeout_ns it gives up, writes 0 to *result (device int32), records device error 1 and
 * returns; the context stays usable. */
int moe_selftest_bounded_wait(uint64_t timeout_ns, int32_t* result, void* stream);

/* Measurement aid (no counterpart in the reference): writes zeros over `bytes` bytes at dst
 * (16-byte aligned, bytes a multiple of 16) with 16-byte stores from 8 blocks per SM, the
 * access size of the GEMM epilogues.  bench.py times it to measure this part's DRAM write
 * bandwidth, a bound of the weight-gradient GEMM. */
int moe_write_probe(void* dst, size_t bytes, void* stream);

/* ---------------------------------------------------------------- top-k softmax
 * Replaces tg::fused_topk_softmax_fwd
 * (triton_gmm_ops/fused_topk_softmax_ops.py:121-138, kernel :17-70).
 * logits [T, E] (dtype), weights [T, K] (same dtype), indices [T, K] int32.
 * Top-K by value with ties broken towards the lower expert index, then a softmax
 * over the K selected values computed in fp32. */
int moe_topk_softmax_fwd(const void* logits, int dtype, int64_t num_tokens, int32_t num_experts,
                         int32_t topk, void* weights, int32_t* indices, void* stream);

/* Replaces tg::fused_topk_softmax_bwd (fused_topk_softmax_ops.py:150-165, kernel :83-114).
 * grad_logits [T, E] is fully written: w*(g - sum_k g*w) at the selected experts, 0 elsewhere. */
int moe_topk_softmax_bwd(const void* grad_weights, const void* weights, const int32_t* indices,
                         int dtype, int64_t num_tokens, int32_t num_experts, int32_t topk,
                         void* grad_logits, void* stream);

/* ---------------------------------------------------------------- permute
 * Bytes of device workspace moe_permute needs for these sizes. */
size_t moe_permute_workspace_bytes(int64_t num_tokens, int32_t topk, int32_t num_experts);

/* Replaces tg::permute_countsort (triton_gmm_ops/permute_ops.py:82-110) together with
 * _group_offsets (:36-43).  input [T, C] (dtype), indices [T, K] int32 expert ids.
 * Writes offsets [E+1] (offsets[0]=0, inclusive prefix of the expert histogram),
 * row_id_map [K*T] (row_id_map[k*T + t] = destination row of slot (t,k)) and
 * permuted [num_out, C] with permuted[row_id_map[k*T+t]] = input[t].  Rows are
 * grouped by expert in stable slot order (the order of a stable argsort of the
 * flattened indices).  num_out >= T*K; rows past T*K are left unwritten. */
int moe_permute(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                int32_t topk, int64_t num_cols, int32_t num_experts, int64_t num_out,
                void* permuted, int32_t* row_id_map, int32_t* offsets, void* workspace,
                size_t workspace_bytes, void* stream);

/* moe_permute with token dropping, the capacity case the reference leaves out
 * (triton_gmm_ops/permute_ops.py:89-93 clamps num_out_tokens up to T*K instead).  Slots
 * are ranked inside their expert in stable slot order (slot j = t*K + k: lower token
 * first); a slot is kept while its rank is below `capacity` (<= 0: no per-expert limit)
 * and its output row is below num_out (the rows of `permuted`).  A dropped slot gets
 * row_id_map = -1 and no row; offsets [E+1] count the kept rows only (offsets[E] <=
 * num_out), so grouped GEMMs over them never see a dropped slot, and moe_unpermute_fwd /
 * _bwd treat -1 as an absent slot (it contributes zero; its prob_grad is zero).  Same
 * workspace as moe_permute. */
int moe_permute_capacity(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                         int32_t topk, int64_t num_cols, int32_t num_experts, int32_t capacity,
                         int64_t num_out, void* permuted, int32_t* row_id_map, int32_t* offsets,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Index pass of moe_permute (no rows copied) that also writes the inverse map:
 * row_src[row] = the token whose slot lands in that permuted row ([T*K] int32).  With it
 * the grouped GEMMs can read the permuted operand straight from the token-order input
 * (moe_gmm_*_gather), so the permuted copy is never written: the fused permute -> GEMM of
 * the reference's experiment (develop/experiment/fused_ops.py:31-107, rows fetched through
 * `sorted_id_map`).  row_id_map / offsets as moe_permute; workspace as moe_permute. */
int moe_permute_index(const int32_t* indices, int64_t num_tokens, int32_t topk, int32_t num_experts,
                      int32_t* row_id_map, int32_t* offsets, int32_t* row_src, void* workspace,
                      size_t workspace_bytes, void* stream);

/* SwiGLU between the expert GEMMs: out = silu(gate) * up over n elements, replacing the
 * reference layer's `F.silu(gate) * up` (tests/test_moe.py:82) and its autograd backward.
 * Rounding follows those PyTorch passes: silu rounded to dtype, then the product. */
int moe_swiglu_fwd(const void* gate, const void* up, void* out, int64_t n, int dtype, void* stream);
/* grad_gate = silu'(gate) * rnd(grad_out * up), grad_up = grad_out * rnd(silu(gate)). */
int moe_swiglu_bwd(const void* grad_out, const void* gate, const void* up, void* grad_gate,
                   void* grad_up, int64_t n, int dtype, void* stream);

/* Copy step of moe_permute with a caller-supplied map: out[row_id_map[k*T+t]] = input[t]
 * for every k (input [T, C], out rows as many as the map names).  This is the copy of the
 * reference's permute scatter (permute_ops.py:50-74) without the counting sort; it is also
 * the backward of permute_backward with K = 1. */
int moe_scatter_rows(const void* input, int dtype, const int32_t* row_id_map, int64_t num_tokens,
                     int32_t topk, int64_t num_cols, void* out, void* stream);

/* No counterpart in the reference.  moe_permute for callers that cannot allocate device
 * memory at call time (work recorded into a stream capture or run from inside an
 * allocator, runtimes that plan all memory ahead, fixed device arenas): the per-tile
 * expert counts live in a 1 MiB array inside the library instead of in a workspace
 * argument.  Same outputs and contract as moe_permute; the caller still passes inputs and
 * outputs.  Sizes whose counts (ceil(T*K / 512) * E int32) exceed the array are rejected
 * with MOE_ERR_INVALID_ARG; moe_permute_noalloc_max_slots(E) gives the largest T*K.
 * The first call on a device looks up the array's device address (make it before any
 * stream capture).  All calls share the one array: calls that overlap on the GPU (on
 * different streams) race and must be serialised by the caller.  Calls no allocator. */
int moe_permute_noalloc(const void* input, int dtype, const int32_t* indices, int64_t num_tokens,
                        int32_t topk, int64_t num_cols, int32_t num_experts, int64_t num_out,
                        void* permuted, int32_t* row_id_map, int32_t* offsets, void* stream);
size_t moe_permute_noalloc_max_slots(int32_t num_experts);

/* ---------------------------------------------------------------- unpermute
 * Replaces tg::unpermute_forward (triton_gmm_ops/unpermute_ops.py:58-72, kernel :20-55).
 * out[t] = sum_k prob[t,k] * input[row_id_map[k*T+t]], accumulated in fp32 in k order
 * (product rounded, then sum rounded), cast to dtype.  prob [T, K] of prob_dtype.
 * A NULL prob means prob == 1 everywhere: this is permute_backward
 * (triton_gmm_ops/permute_ops.py:130-133). */
int moe_unpermute_fwd(const void* input, int dtype, const int32_t* row_id_map, const void* prob,
                      int prob_dtype, int64_t num_tokens, int32_t topk, int64_t num_cols, void* out,
                      void* stream);

/* Replaces tg::unpermute_backward (unpermute_ops.py:153-172, kernel :93-150).
 * act_grad[row_id_map[k*T+t]] = cast(prob[t,k] * grad_out[t]) and
 * prob_grad[t,k] = sum_c grad_out[t,c] * input_fwd[row_id_map[k*T+t], c] (fp32, cast to
 * prob_dtype).  Rows of act_grad that row_id_map does not name are left unwritten. */
int moe_unpermute_bwd(const void* grad_out, const void* input_fwd, int dtype,
                      const int32_t* row_id_map, const void* prob, int prob_dtype,
                      int64_t num_tokens, int32_t topk, int64_t num_cols, void* act_grad,
                      void* prob_grad, void* stream);

/* ---------------------------------------------------------------- grouped GEMM
 * Replaces tg::gmm_tma_fwd_raw / group_gemm_tma_fn
 * (triton_gmm_ops/grouped_gemm_ops_sm90.py:151-202) and tg::gmm_fwd_raw
 * (triton_gmm_ops/grouped_gemm_ops.py:75-101).
 * A [M_total, K]; B [E, N, K] if trans_b else [E, K, N]; C [M_total, N].
 * C[rows of e] = A[rows of e] @ (B[e]^T if trans_b else B[e]), fp32 accumulation.
 * bf16/fp16 run on the tcgen05 tensor-core kernel; fp32 (and shapes whose rows are not
 * 16-byte multiples) on a CUDA-core kernel with fp32 FMA. */
int moe_gmm_fwd(const void* A, const void* B, void* C, const int32_t* offsets,
                int32_t num_offsets, int64_t m_total, int64_t n, int64_t k, int32_t num_experts,
                int trans_b, int dtype, void* stream);

/* dgrad of moe_gmm_fwd, the grad_A branch of GroupedGEMMAutogradSM90.backward
 * (grouped_gemm_ops_sm90.py:224-233).  grad_C [M_total, N] -> grad_A [M_total, K].
 * Reads B in place for both values of trans_b (no transposed weight copy). */
int moe_gmm_dgrad(const void* grad_C, const void* B, void* grad_A, const int32_t* offsets,
                  int32_t num_offsets, int64_t m_total, int64_t n, int64_t k,
                  int32_t num_experts, int trans_b, int dtype, void* stream);

/* grad_A = grad_C1 . op(B1[e]) + grad_C2 . op(B2[e]) per expert row range in ONE launch: the
 * two contractions run as consecutive segments into one fp32 accumulator, rounded once.
 * grad_C1 [m_total, n1], grad_C2 [m_total, n2], B1 / B2 laid out as moe_gmm_dgrad's B
 * (n1 / n2 in place of n), grad_A [m_total, k].  This is the input gradient of the gate and
 * up projections of a SwiGLU MLP (dgrad(dgate, W_gate) + dgrad(dup, W_up)), which the
 * reference forms with two grouped GEMMs and an add (its layer's autograd through
 * triton_gmm_ops/grouped_gemm_ops_sm90.py:224-233 twice).  Tensor-core path only: 16-bit
 * operands, 16-byte aligned pointers, n1, n2, k multiples of 8; MOE_ERR_INVALID_ARG
 * otherwise (call moe_gmm_dgrad twice and add). */
int moe_gmm_dgrad_dual(const void* grad_C1, const void* B1, const void* grad_C2, const void* B2,
                       void* grad_A, const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                       int64_t n1, int64_t n2, int64_t k, int32_t num_experts, int trans_b,
                       int dtype, void* stream);

/* wgrad of moe_gmm_fwd: replaces tg::gmm_bwd_B_raw (grouped_gemm_ops.py:174-192).
 * grad_B [E, N, K] if trans_b else [E, K, N] (the reference supports trans_b only);
 * experts with no rows get zeros. */
int moe_gmm_wgrad(const void* A, const void* grad_C, void* grad_B, const int32_t* offsets,
                  int32_t num_offsets, int64_t m_total, int64_t n, int64_t k,
                  int32_t num_experts, int trans_b, int dtype, void* stream);

/* Gathered-A forms (permute fused into the GEMM, develop/experiment/fused_ops.py:31-107 and
 * its weight gradient): row r of A is row a_rows[r] of A_src [a_src_rows, k] (a_rows from
 * moe_permute_index), fetched with TMA gather4, so the permuted copy of A is never
 * materialised.  Results equal moe_gmm_fwd / moe_gmm_gate_up_fwd / moe_gmm_wgrad on the
 * materialised permuted A bit for bit.  Tensor-core path only (16-bit, 16-byte aligned,
 * sizes multiples of 8; MOE_ERR_INVALID_ARG otherwise); wgrad_gather takes trans_b only. */
int moe_gmm_fwd_gather(const void* A_src, const int32_t* a_rows, int64_t a_src_rows, const void* B,
                       void* C, const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                       int64_t n, int64_t k, int32_t num_experts, int trans_b, int dtype,
                       void* stream);
int moe_gmm_gate_up_fwd_gather(const void* A_src, const int32_t* a_rows, int64_t a_src_rows,
                               const void* B_gate, const void* B_up, void* gate, void* up, void* h,
                               const int32_t* offsets, int32_t num_offsets, int64_t m_total,
                               int64_t n, int64_t k, int32_t num_experts, int trans_b, int dtype,
                               void* stream);
int moe_gmm_wgrad_gather(const void* A_src, const int32_t* a_rows, int64_t a_src_rows,
                         const void* grad_C, void* grad_B, const int32_t* offsets,
                         int32_t num_offsets, int64_t m_total, int64_t n, int64_t k,
                         int32_t num_experts, int trans_b, int dtype, void* stream);

/* Gate and up projections of a SwiGLU expert layer with the SwiGLU applied, in one launch:
 *   gate = A @ B_gate[e]^T, up = A @ B_up[e]^T (trans_b; else A @ B[e]),
 *   h = rnd(rnd(silu(gate)) * up)
 * over the rows of each expert; B_gate / B_up as B of moe_gmm_fwd, gate / up / h
 * [M_total, N].  The three outputs equal two moe_gmm_fwd calls followed by moe_swiglu_fwd
 * bit for bit; gate and up are kept for the backward.  Replaces the reference layer's
 * two grouped_gemm calls and `F.silu(gate) * up` (tests/test_moe.py:80-82). */
int moe_gmm_gate_up_fwd(const void* A, const void* B_gate, const void* B_up, void* gate,
                        void* up, void* h, const int32_t* offsets, int32_t num_offsets,
                        int64_t m_total, int64_t n, int64_t k, int32_t num_experts, int trans_b,
                        int dtype, void* stream);

/* Backward through the down projection and the SwiGLU of a SwiGLU expert layer, in one
 * launch: dh = moe_gmm_dgrad(grad_C, B) ([M_total, K], rounded to dtype), then
 *   grad_gate, grad_up = moe_swiglu_bwd(dh, gate, up)
 * with gate / up [M_total, K] the forward's projections.  Both results equal the two
 * separate calls bit for bit; dh itself is never written.  Replaces the down GEMM's dgrad
 * and the autograd backward of `F.silu(gate) * up` in the reference layer
 * (tests/test_moe.py:82-83). */
int moe_gmm_dgrad_swiglu_bwd(const void* grad_C, const void* B, const void* gate, const void* up,
                             void* grad_gate, void* grad_up, const int32_t* offsets,
                             int32_t num_offsets, int64_t m_total, int64_t n, int64_t k,
                             int32_t num_experts, int trans_b, int dtype, void* stream);

/* ---------------------------------------------------------------- expert parallelism over peer memory
 * No counterpart in the reference, which has no multi-GPU path: the dispatch and combine of
 * an expert-parallel layer, moving rows between the GPUs' buffers over NVLink in place of
 * an all-to-all.  Rank r owns experts [r*El, (r+1)*El).  `bases` / `in_bases` /
 * `act_bases` / `flags` are DEVICE arrays of `world` pointers: entry r is rank r's buffer as
 * mapped in this process (this rank's own allocation, or a peer's opened with
 * moe_ipc_open).  Every row a kernel touches is checked against the receive capacity first;
 * a bad slot is skipped and raises device error 3. */

/* cudaMalloc of `bytes` plus its CUDA IPC handle (64 bytes written to `handle`), for a
 * buffer the peers map with moe_ipc_open. */
int moe_ipc_malloc(size_t bytes, void** ptr, void* handle);
/* Maps a peer's buffer (its 64-byte IPC handle) into this process. */
int moe_ipc_open(const void* handle, void** ptr);
int moe_ipc_close(void* ptr);
int moe_ipc_free(void* ptr);

/* Destination of every slot: slot j = k*T + t with expert e = indices[t*K+k] goes to rank
 * e / experts_per_rank at row row_id_map[j] + delta[e] (row_id_map from moe_permute over
 * the global experts; delta[e] places this rank's rows of expert e in the owner's receive
 * buffer).  ranks[j] = -1 (and device error 3) when e or the row is out of range. */
int moe_ep_slot_map(const int32_t* indices, const int32_t* row_id_map, const int32_t* delta,
                    int64_t num_tokens, int32_t topk, int32_t num_experts,
                    int32_t experts_per_rank, int32_t world, int64_t capacity, int32_t* ranks,
                    int32_t* rows, void* stream);
/* Dispatch: input row t to bases[ranks[j]] row rows[j] for each of its K slots (the
 * permute copy with peer destinations).  `status` (device int32, nullable) is the barrier
 * status of moe_ep_barrier: when it reads 0 the kernel stores nothing (a peer that missed a
 * barrier may still be reading its buffers).  The same holds for the two combines below,
 * which then read no peer row (those slots contribute zero). */
int moe_ep_dispatch(const void* input, int dtype, void* const* bases, const int32_t* ranks,
                    const int32_t* rows, int64_t num_tokens, int32_t topk, int64_t num_cols,
                    const int32_t* status, void* stream);
/* Combine: out[t] = sum_k prob[t,k] * row(slot k of t) read from bases[ranks[j]], with the
 * rounding of moe_unpermute_fwd; prob NULL means 1 (the dispatch's backward). */
int moe_ep_combine(const void* const* bases, int dtype, const int32_t* ranks, const int32_t* rows,
                   const void* prob, int prob_dtype, int64_t num_tokens, int32_t topk,
                   int64_t num_cols, void* out, const int32_t* status, void* stream);
/* Combine backward (moe_unpermute_bwd over peer rows): act row of slot j (in act_bases) =
 * grad_out[t] * prob[t,k]; prob_grad[t,k] = <grad_out[t], row of slot j in in_bases>. */
int moe_ep_combine_bwd(const void* grad_out, const void* const* in_bases, void* const* act_bases,
                       int dtype, const int32_t* ranks, const int32_t* rows, const void* prob,
                       int prob_dtype, int64_t num_tokens, int32_t topk, int64_t num_cols,
                       void* prob_grad, const int32_t* status, void* stream);
/* dst[r] += src[r] (fp32 sum rounded to dtype) for rows r < min(*n_rows, max_rows) of two
 * [max_rows, num_cols] buffers; n_rows is a device int32 (e.g. the last grouped-GEMM
 * offset), so worst-case-sized buffers cost only their live rows. */
int moe_add_rows(void* dst, const void* src, const int32_t* n_rows, int64_t max_rows,
                 int64_t num_cols, int dtype, void* stream);
/* Cross-GPU barrier on `world` int64 flag arrays of `world` slots each (one per rank, in
 * IPC memory).  The barrier's epoch is *epoch_counter + 1 (a device int64 of this rank,
 * written back by the barrier, so a launch captured in a CUDA graph advances it on every
 * replay; start it at 0 with the flags zeroed).  Writes the epoch to slot `rank` of every
 * rank's array (after a system-scope fence), then waits until every slot of this rank's
 * array reaches it.  Gives up after timeout_ns: *status (device int32, may be NULL) = 0 and
 * device error 4; a barrier that completes leaves *status unchanged, so one status word
 * records any failure over many barriers.  Every rank must run the same sequence of
 * barriers.  The ranks must run on different GPUs. */
int moe_ep_barrier(int64_t* const* flags, int32_t rank, int32_t world, int64_t* epoch_counter,
                   uint64_t timeout_ns, int32_t* status, void* stream);
/* Counts exchange of the peer-memory layout: counts[0..E) of this rank go to row `rank` of
 * every rank's [world, E] int32 array (bases[r] is rank r's, mapped here).  A barrier must
 * follow before any rank reads its array; no rank may write again before every rank has
 * read (the layer's later barriers order that). */
int moe_ep_put_counts(const int32_t* counts, int32_t num_experts, int32_t* const* bases,
                      int32_t rank, int32_t world, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MOE_B200_H_ */
