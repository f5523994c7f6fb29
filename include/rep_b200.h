/*
 * rep_b200.h -- C ABI of the B200 (sm_100a) RepEncoder W8A8 hot path.
 *
 * Plain pointers and sizes only; every device pointer refers to memory of the
 * current CUDA device, and every call is asynchronous on `stream` (a
 * cudaStream_t passed as void*; NULL = legacy default stream).  Calls return
 * an rb_status; rb_last_error() gives the message of the last failure on the
 * calling thread.  The library never allocates device memory.
 *
 * Each entry point names the reference interface it replaces (paths inside
 * YuDeng0102/baidu_cti_grab).
 */
#ifndef REP_B200_H
#define REP_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
enum rb_dtype { RB_F32 = 0, RB_BF16 = 1, RB_F16 = 2, RB_I32 = 3, RB_I8 = 4, RB_I64 = 5 };

/* activation quantisation: dynamic per-token, static per-tensor, or none (LayerNorm output only) */
enum rb_act_mode { RB_ACT_DYNAMIC = 0, RB_ACT_STATIC = 1, RB_ACT_NONE = 2 };

/* return codes; the Python layer maps them to the reference's exception types */
enum rb_status {
  RB_OK = 0,
  RB_ERR_VALUE = 1,       /* bad shape / argument  -> ValueError */
  RB_ERR_UNSUPPORTED = 2, /* valid but not supported by this library -> ValueError */
  RB_ERR_CUDA = 3,        /* CUDA runtime/driver error -> RuntimeError */
  RB_ERR_DEVICE = 4       /* not an sm_100 device, or a device-side timeout -> RuntimeError */
};

/* maximum number of slots one call of the gather kernel takes */
#define RB_MAX_SLOTS 32
#define RB_MAX_DEST 8 /* ranks a pooled-row scatter can address */

const char* rb_last_error(void);
int rb_version(void);

/* 1 when the current device is sm_100 and the library's kernels can launch on it. */
int rb_device_supported(void);

/*
 * Device-side watchdog status: 0, or the code of the first bounded wait that
 * ran out of time in one of this library's kernels since the last reset
 * (kernels return instead of hanging).  Synchronous; reset=1 clears it.
 */
int rb_device_error(int reset);

/* Test hook: run the GEMM pipeline's bounded mbarrier wait on a barrier that
 * nothing arrives on, with a budget of `budget_ns`; sets the watchdog status. */
int rb_selftest_wait_timeout(uint64_t budget_ns, void* stream);

/*
 * Fused gather -> sum-pool -> concat -> LayerNorm -> int8 quantisation.
 * Replaces models.py:24-48 (RepEncoder.forward: 28x clamp + nn.EmbeddingBag
 * (mode='sum', padding_idx=0) + torch.cat + nn.LayerNorm) followed by
 * quantization/w8a8_triton_kernels.py:392-460 (quantize_activation, dynamic
 * per-token or static per-tensor), without writing the concatenated row.
 *
 *   table            [num_rows, emb_dim] row-major, table_dtype RB_BF16 or RB_F32;
 *                    emb_dim must be 512.  Ids are clamped to [0, num_rows-1]
 *                    and id 0 is the padding row (excluded from the sum).
 *   slot_values[s]   device int64 ids of slot s (nnz[s] of them)
 *   slot_offsets[s]  device int64 [num_items+1]; bag i = [off[i], off[i+1]) for
 *                    i < num_items-1 and [off[num_items-1], nnz[s]) for the last
 *                    (the reference passes offsets[:-1]); ends clamp to nnz[s].
 *   slot_nnz         host array [num_slots]
 *   ln_gamma/ln_beta [num_slots*512] in ln_dtype (RB_BF16/RB_F32/RB_F16), eps
 *   act_mode         RB_ACT_DYNAMIC: q_out + scale_out[num_items] (fp32)
 *                    RB_ACT_STATIC:  q_out with 1/static_scale[0]
 *                    RB_ACT_NONE:    no quantisation (ln_out required)
 *   q_out            int8 [num_items, ldq] (ldq >= num_slots*512, multiple of 16)
 *   pooled_out, ln_out  optional [num_items, num_slots*512] in table_dtype.
 * The LayerNorm and the int8 values are computed in the row dtype (= table dtype).
 */
int rb_rep_gather_ln_quant(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                           const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                           const int64_t* slot_nnz, int num_slots, int64_t num_items,
                           const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                           int act_mode, const void* static_scale, int static_scale_dtype,
                           int8_t* q_out, int64_t ldq, float* scale_out, void* pooled_out,
                           void* ln_out, void* stream);

/*
 * rb_rep_gather_ln_quant with the width of the ids and offsets as a parameter:
 * index_dtype RB_I64 (the reference's collate output, models.py:27-34 reads
 * int64 `values`/`offsets`) or RB_I32 (half the bytes to pack, copy and read;
 * valid while ids, offsets and nnz stay below 2^31, e.g. a table of fewer than
 * 2^31 rows).  slot_values[s] / slot_offsets[s] point to arrays of that type;
 * everything else, the arithmetic included, is as in rb_rep_gather_ln_quant.
 */
int rb_rep_gather_ln_quant_idx(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                               int index_dtype, const void* const* slot_values, const void* const* slot_offsets,
                               const int64_t* slot_nnz, int num_slots, int64_t num_items,
                               const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                               int act_mode, const void* static_scale, int static_scale_dtype,
                               int8_t* q_out, int64_t ldq, float* scale_out, void* pooled_out,
                               void* ln_out, void* stream);

/*
 * Gather + sum-pool only (models.py:27-34, the 28 nn.EmbeddingBag calls), for
 * a subset of slots, writing pooled rows [num_items, ldp] (row dtype = table
 * dtype) with slot j of the call at columns [col_slot[j]*512, +512).  Used by
 * the slot-sharded multi-GPU path before the pooled-row exchange.
 */
int rb_rep_gather_pool(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                       const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                       const int64_t* slot_nnz, const int* col_slot, int num_slots,
                       int64_t num_items, void* pooled_out, int64_t ldp, void* stream);

/*
 * rb_rep_gather_pool whose output rows go straight to the ranks that own the
 * items (the pooled-row exchange of the slot-sharded multi-GPU path, done by
 * the pooling kernel itself with stores over NVLink): item i, with
 * dest_begin[d] <= i < dest_begin[d+1], is written at
 * dest[d] + (i - dest_begin[d])*ld + col_slot[s]*512 (elements).  dest[d] may
 * be another GPU's memory mapped into this process (rb_ipc_import); dest_begin
 * holds num_dest+1 nondecreasing item indices from 0 to num_items; dest rows
 * must be 32-byte aligned (ld*2 a multiple of 32 bytes) for bf16 tables.  The
 * caller hands the rows over with a barrier on the same stream after the call,
 * e.g. an NCCL all-reduce: the kernel's stores happen before its completion,
 * and the barrier's cross-GPU release/acquire publishes them to the owners.
 * Items are taken in the order item_shift, item_shift+1, ... (mod num_items):
 * ranks that start at different owners' ranges keep every NVLink busy instead
 * of all storing into one owner at a time.  The pooling follows models.py:27-34;
 * the exchange has no counterpart in the reference, which runs on one GPU.
 */
int rb_rep_gather_pool_scatter(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                               const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                               const int64_t* slot_nnz, const int* col_slot, int num_slots, int64_t num_items,
                               void* const* dest, const int64_t* dest_begin, int num_dest, int64_t ld,
                               int64_t item_shift, void* stream);

/*
 * CUDA IPC for the scatter's destinations (no counterpart in the reference).
 * rb_ipc_export: a 64-byte handle (RB_IPC_HANDLE_BYTES) for the device
 * allocation that holds ptr, and ptr's byte offset in it.  rb_ipc_import, in
 * another process on the same node: the pointer at that offset of the mapped
 * allocation (peer access enabled).  rb_ipc_close(ptr, offset) unmaps it.
 */
#define RB_IPC_HANDLE_BYTES 64
int rb_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int rb_ipc_import(const void* handle, int64_t offset, void** ptr_out);
int rb_ipc_close(void* ptr, int64_t offset);

/*
 * LayerNorm + int8 quantisation of dense pooled rows x[num_items, ldx]
 * (x_dtype, width num_slots*512): the part of rb_rep_gather_ln_quant after the
 * gather (models.py:45 + w8a8_triton_kernels.py:392-460), with the same
 * arithmetic.  RB_ACT_NONE writes only ln_out (kernels/rep_encoder_fusion.py:6-30
 * LayerNorm for the unquantised LN+Linear path).
 */
int rb_layernorm_quant(const void* x, int x_dtype, int64_t num_items, int num_slots, int64_t ldx,
                       const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                       int act_mode, const void* static_scale, int static_scale_dtype,
                       int8_t* q_out, int64_t ldq, float* scale_out, void* ln_out, void* stream);

/*
 * rb_layernorm_quant with each slot's 512 columns read from its own place:
 * slot s of item i at slot_rows[s] + i*ld (elements).  Lets the slot-sharded
 * multi-GPU path normalise the rows it received from every rank in place
 * (models.py:39-45 concat + LayerNorm, without materialising the concat).
 */
int rb_layernorm_quant_slots(const void* const* slot_rows, int x_dtype, int64_t num_items, int num_slots,
                             int64_t ld, const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                             int act_mode, const void* static_scale, int static_scale_dtype, int8_t* q_out,
                             int64_t ldq, float* scale_out, void* ln_out, void* stream);

/* quantization/w8a8_triton_kernels.py:41-64,392-422 dynamic_per_token_quantize_activation[_out]:
 * x[M,K] (row stride ldx elements) -> q[M,K] (row stride ldq), scale[M] fp32. */
int rb_quant_dynamic_per_token(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx,
                               int8_t* q, int64_t ldq, float* scale, void* stream);

/* quantization/w8a8_triton_kernels.py:23-38,375-389 static_quantize_activation[_out]:
 * contiguous x[numel] with per-tensor scale[0] (scale_dtype RB_F32/RB_BF16/RB_F16). */
int rb_quant_static(const void* x, int x_dtype, int64_t numel, const void* scale, int scale_dtype,
                    int8_t* q, void* stream);

/* kernels/quantization.py:6-35,243-278 quantize_rows_int8_triton (v1 rounding):
 * x[M,K] -> q[M,K] in [-127,127], scale[M] = max(amax/127, 1e-8). */
int rb_quant_rows_v1(const void* x, int x_dtype, int64_t M, int64_t K, int64_t ldx, int8_t* q,
                     int64_t ldq, float* scale, void* stream);

/* quantization/w8a8_preprocess.py:46-57 quantize_weight_per_channel:
 * w[N,K] (w_dtype, row stride ldw) -> q[N,K] int8 (round half to even) and scale[N] fp32. */
int rb_quantize_weight_per_channel(const void* w, int w_dtype, int64_t N, int64_t K, int64_t ldw,
                                   int8_t* q, float* scale, void* stream);

/* Repack a [K,N] int8 weight view with element strides (stride_k, stride_n) into
 * the GEMM's K-contiguous [N,K] layout (quantization_utils.py:21 stores qweight_t
 * row-major [K,N]; w8a8_preprocess.py:54 makes it a transposed view). */
int rb_pack_weight_nk(const int8_t* src, int64_t K, int64_t N, int64_t stride_k, int64_t stride_n,
                      int8_t* dst, void* stream);

/*
 * W8A8 GEMM: acc[m,n] = sum_k A[m,k] * B[n,k] (int32, exact), then
 *   out = ((f32(acc) * sa) * sb[n]) + bias[n]      stored as out_dtype
 * or the raw int32 acc when out_dtype == RB_I32 (scales/bias ignored).
 * Replaces quantization/w8a8_triton_kernels.py:174-318,470-640
 * (w8a8_scaled_mm[_out], int8_mm_no_scale[_out]) and kernels/quantization.py:38-105
 * (_w8a8_matmul_kernel).  tcgen05 kind::i8 on sm_100a with the accumulator in TMEM
 * (one-SM tiles; CTA-pair tiles for M >= 4096); M <= 16 uses int8 dot products
 * on the CUDA cores (one launch), with the same results bit for bit.
 *   A     int8 [M, lda]  (K contiguous; lda % 16 == 0, 16-byte aligned)
 *   B     int8 [N, ldb]  (K contiguous; ldb % 16 == 0, 16-byte aligned)
 *   sa    per-row [M] (sa_per_row=1) or scalar [1]; sa_dtype RB_F32/RB_BF16/RB_F16
 *   sb    [N], sb_dtype; bias [N] bias_dtype or NULL
 *   out   [M, ldo] out_dtype RB_BF16 / RB_F16 / RB_F32 / RB_I32
 */
int rb_w8a8_gemm(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                 int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb,
                 int sb_dtype, const void* bias, int bias_dtype, void* out, int64_t ldo,
                 int out_dtype, void* stream);

/*
 * rb_w8a8_gemm with a caller-provided int32 workspace: for mid M (from 257 rows
 * while the one-SM kernel's 128 x 256 tiles are fewer than the SMs, and from
 * 2048 rows while the two-SM kernel's 256 x 256 tiles cover at most half of the
 * CTA pairs; M up to 4608 at N = 512) the K dimension is split across
 * CTAs, each split's int32 partial goes to the workspace, and a second kernel
 * sums the splits (int32 addition is exact in any order) and applies the
 * epilogue.  Same results as rb_w8a8_gemm,
 * bit for bit.  rb_w8a8_gemm_workspace_size(M, N, K) gives the number of int32
 * elements needed (0: no split for this shape); a smaller workspace runs unsplit.
 * Replaces the same reference interfaces as rb_w8a8_gemm.
 */
int64_t rb_w8a8_gemm_workspace_size(int64_t M, int64_t N, int64_t K);
int rb_w8a8_gemm_ws(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                    int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb, int sb_dtype,
                    const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                    int32_t* workspace, int64_t workspace_elems, void* stream);

/*
 * rb_w8a8_gemm together with the transformer's first LayerNorm
 * (models.py:216-217: layer 0 begins residual = x; x = norm1[0](x), x being
 * the RepEncoder output this GEMM produces): below M = 4096 one kernel with the
 * LayerNorm in the GEMM's epilogue, from M = 4096 the GEMM followed by a
 * LayerNorm pass over its output on the same stream (measured faster there;
 * the bits are the same either way).  out is rb_w8a8_gemm's result
 * (the residual), ln_out = LayerNorm(out) over the 512 columns with
 * ln_gamma/ln_beta (ln_dtype RB_F32/RB_BF16/RB_F16) and eps, in the reduction
 * order of ATen's CUDA LayerNorm, so it equals nn.LayerNorm on out bit for
 * bit.  N must be 512; out and ln_out share out_dtype (RB_BF16/RB_F16/RB_F32);
 * sb and bias 16-byte aligned.  Replaces quantization/w8a8_triton_kernels.py's
 * scaled GEMM (:470-564) followed by the first norm1 of models.py:217.
 */
int rb_w8a8_gemm_ln(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                    int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb, int sb_dtype,
                    const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                    const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps, void* ln_out,
                    int64_t ldl, void* stream);

/*
 * Unquantised Linear on the tensor cores: out[m,n] = sum_k A[m,k] * B[n,k] + bias[n].
 * Replaces the GEMM of kernels/rep_encoder_fusion.py:33-112 (_layernorm_linear_kernel,
 * a tl.dot of bf16 operands -- or fp32 operands, which Triton multiplies as tf32 --
 * with fp32 accumulation, then + bias) behind layernorm_linear_triton (:169-243).
 *   A   [M, lda], B [N, ldb]: both RB_BF16 (tcgen05 kind::f16) or both RB_F32
 *       (kind::tf32); K contiguous.  16-byte aligned bases and row pitches take
 *       the TMA / tensor-core path; other layouts a CUDA-core kernel.
 *   accumulators fp32 (TMEM), bias [N] f32/bf16/f16 or NULL added in fp32,
 *   out [M, ldo] RB_BF16 / RB_F16 / RB_F32.
 * Floating-point sums: results agree with an fp32 matmul of the same operands
 * to within fp32 accumulation error (tf32 rounding of the operands for f32).
 */
int rb_fp_gemm(const void* A, int ab_dtype, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
               int64_t K, const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
               void* stream);

/*
 * rb_w8a8_gemm_ws for callers that cannot allocate device memory themselves
 * (their device memory belongs to another allocator's pool or a pre-sized
 * arena, or their host forbids cudaMalloc after start-up).  No counterpart in
 * the reference.  The split-K workspace comes from a fixed 20 MiB device array in
 * the library (held on every GPU that loads it); shapes needing more are
 * rejected with RB_ERR_VALUE.  The first call on a device resolves the array's
 * address and keeps it once resolved (make that call before any stream
 * capture).  Calls share the array, so
 * calls that overlap on the GPU race; no state carries from one call to the
 * next.  Same results as rb_w8a8_gemm, bit for bit; allocates nothing.
 */
int rb_w8a8_gemm_noalloc(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                         int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb, int sb_dtype,
                         const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype, void* stream);

/*
 * The SMoE expert layer after the gate (models.py:131-178: sort the routed
 * entries by expert, pack, two bmm's with the stacked expert weights, relu,
 * score weighting, index_add_), without a host read of the per-expert counts
 * (models.py:160) and without padding rows.
 *   x          [T, ldx] RB_BF16 or RB_F16 (the model dtype), d_model = D
 *   topk_idx   [T, k] contiguous, RB_I64 (torch.topk's output) or RB_I32,
 *              expert ids in [0, E); an id outside it adds nothing and sets
 *              the device error word (rb_device_error)
 *   topk_score [T, k] contiguous gate scores in the model dtype
 *   w1 [E, F, D], b1 [E, F] or NULL (each expert's fc1 nn.Linear weight and
 *   bias, stacked), w2 [E, D, F], b2 [E, D] or NULL (fc2), all in the model
 *   dtype; D and F multiples of 64, E <= 64
 *   workspace  rb_smoe_workspace_size(T, k, E, D, F, x_dtype) bytes, 256-byte aligned
 *   out        [T, ldo], 32-byte aligned rows; every row written
 * Each expert output is rounded to the model dtype where the reference's
 * torch ops round (bmm, + bias, * score, the index_add_ sum); the fp32
 * accumulation order inside the dot products is this library's own.
 * rb_smoe_workspace_size returns -1 for an invalid shape or dtype.
 */
int64_t rb_smoe_workspace_size(int64_t T, int k, int E, int D, int F, int x_dtype);
int rb_smoe_experts(const void* x, int x_dtype, int64_t ldx, int64_t T, int D, const void* topk_idx,
                    int idx_dtype, const void* topk_score, int k, int E, const void* w1, const void* b1,
                    const void* w2, const void* b2, int F, void* workspace, int64_t workspace_bytes,
                    void* out, int64_t ldo, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* REP_B200_H */
