/*
 * awqb200.h - C ABI of the B200 (sm_100a) AWQ W4A16 quantized-linear library.
 *
 * Every entry point is plain C: device pointers, sizes, a dtype code and a
 * CUDA stream passed as void* (cudaStream_t). Each returns 0 on success or a
 * non-zero status; awqb_last_error() then holds a message for the calling
 * thread. No entry point allocates device memory or synchronises the device
 * unless its comment says so, so the GEMM paths can be captured in CUDA graphs.
 *
 * Status codes:
 *   0 ok, 1 invalid argument, 2 unsupported shape/config, 3 CUDA error,
 *   4 NCCL error, 5 a bounded device-side wait gave up.
 *
 * Each declaration cites the reference (SGLite) interface it replaces, by path
 * inside python/sglite/.
 */
#ifndef AWQB200_H
#define AWQB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AWQB_ABI_VERSION 1

enum { AWQB_DTYPE_F16 = 0, AWQB_DTYPE_BF16 = 1 };

/* Message describing the last failure on this thread ("" if none).
 * Replaces host::PanicError messages, kernels/csrc/include/sglite/utils.h:42-92. */
const char* awqb_last_error(void);
int awqb_abi_version(void);

/* ------------------------------------------------------------------------
 * Weight repack (load time).
 * Replaces awq_marlin_repack + marlin_permute_scales + awq_to_marlin_zero_points
 * called from AWQMarlinLinearMethod.process_weights_after_loading,
 * srt/model_executor/layers/quantization/awq_marlin.py:270-334.
 *
 * AWQ inputs (awq.py:87-124): qweight int32 [batch][K][N/8], qzeros int32
 * [batch][K/G][N/8], scales (fp16 or bf16 bits) [batch][K/G][N]. batch > 1
 * repacks stacked MoE experts ([E, K, N/8], weight_loader.py:134-142).
 * G must be 32, 64 or a multiple of 128, K % G == 0, N % 8 == 0.
 */
int awqb_blob_bytes(int64_t K, int64_t N, int64_t G, int64_t* bytes);
int awqb_repack(const int32_t* qweight, const int32_t* qzeros, const uint16_t* scales,
                int64_t batch, int64_t K, int64_t N, int64_t G, void* blob, void* stream);
/* Exact inverse of awqb_repack (used to prove the repack is lossless). */
int awqb_unrepack(const void* blob, int64_t batch, int64_t K, int64_t N, int64_t G,
                  int32_t* qweight, int32_t* qzeros, uint16_t* scales, void* stream);
/* W[batch][K][N] = (q - z) * s in the activation dtype, with the GEMM's own
 * dequantisation routine; bit-exact with the reference unpack + dequantise,
 * layers/quantization/awq_triton.py:53-62,94-96,119-122. */
int awqb_dequant(const void* blob, int64_t batch, int64_t K, int64_t N, int64_t G, int dtype,
                 void* w, void* stream);

/* ------------------------------------------------------------------------
 * W4A16 GEMM: y[M][N] = x[M][K] * dequant(blob)[K][N] (+ bias[N]).
 * Replaces awq_gemm_triton, layers/quantization/awq_triton.py:144-195 (called by
 * AWQLinearMethod.apply_weights, awq.py:126-147) and gptq_marlin_gemm through
 * apply_awq_marlin_linear, marlin_utils.py:355-415.
 * x, y, bias are in the activation dtype; x 16-byte aligned, rows contiguous.
 * fp32 accumulation. The workspace (size from awqb_gemm_workspace_bytes) must
 * be 256-byte aligned. Its first 8 KiB hold split-tile counters: zero them
 * before the first use; every call leaves them zero again (the rest is scratch
 * for fp32 partial tiles). Calls of any shape may share one workspace as long
 * as it is large enough for each; calls that share it must not overlap in time.
 * At most 1024 CTAs.
 */
int awqb_gemm_workspace_bytes(int64_t M, int64_t K, int64_t N, int64_t G, int64_t* bytes);
int awqb_gemm(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
              const void* blob, const void* bias, void* y, void* workspace,
              int64_t workspace_bytes, void* stream);
/* Same with an explicit token tile (16, 32, 64, 128, 256; 0 = default) and CTA
 * count (0 = one per SM); for tuning and tests. */
int awqb_gemm_workspace_bytes_ex(int64_t M, int64_t K, int64_t N, int64_t G, int ntok,
                                 int64_t ctas, int64_t* bytes);
int awqb_gemm_ex(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                 const void* blob, const void* bias, void* y, void* workspace,
                 int64_t workspace_bytes, int ntok, int64_t ctas, void* stream);
/* The launch awqb_gemm / awqb_gemm_ex would make for these arguments: token
 * tile, CTA count, and cluster size (0 = the small-batch kernel below, one
 * slice of output features per CTA over all of K; 1 = stream-K with the
 * reduction through the workspace; >= 2 = one tile per cluster of that many
 * CTAs, reduced through distributed shared memory). Diagnostics; no
 * counterpart in the reference. */
int awqb_gemm_plan(int64_t M, int64_t K, int64_t N, int64_t G, int ntok, int64_t ctas, int* ntok_out,
                   int64_t* ctas_out, int* cluster_out);

/* Small-batch (decode) kernel that awqb_gemm takes for small M (see
 * awqb_gemm_plan: cluster 0) when no token tile or CTA count is forced: each
 * CTA computes features_per_cta output features over all of K with `warps`
 * compute warps, the weights dequantised in registers and multiplied on
 * mma.sync with fp32 accumulation. Built pairs (features_per_cta, warps):
 * (16, 16), (32, 16), (32, 8), (64, 8); 0 picks by M, N and the SM count.
 * ring (1..16, 0 = by shared memory) is its depth of load stages (warps
 * k-blocks each). 1 <= M <= 32. Needs no workspace. silu_mul != 0 gives the
 * output of awqb_gemm_silu_mul (interleaved gate/up columns, y [M][N/2]).
 * Exposed for tuning and tests. Replaces, for decode batches,
 * awq_gemm_triton, layers/quantization/awq_triton.py:144-195. */
int awqb_gemv_ex(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                 const void* blob, const void* bias, void* y, int features_per_cta, int warps, int ring,
                 int silu_mul, void* stream);

/* GEMM for callers that cannot provide or allocate device memory: a host that
 * owns every device byte through its own arena, or code that must never call
 * cudaMalloc (it may run during CUDA graph capture, or on a path that cannot
 * afford an allocation's implicit synchronisation). No counterpart in the
 * reference. Same computation and arguments as awqb_gemm minus the workspace:
 * the split-K scratch is a fixed array inside the library
 * (awqb_gemm_noalloc_scratch_bytes() = 16 MiB, held by every GPU that loads the
 * library until the process exits). Problems that need more scratch are
 * rejected with status 2 and a message; every M <= 64 fits. Nothing is
 * allocated: the array's device address is looked up once per device by the
 * first call made with that device current, so make that first call before
 * any stream capture. All calls share the one array, so calls that can run at
 * the same time on the GPU (different streams) race and must be serialised by
 * the caller. */
int64_t awqb_gemm_noalloc_scratch_bytes(void);
int awqb_gemm_noalloc(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                      const void* blob, const void* bias, void* y, void* stream);

/* ------------------------------------------------------------------------
 * MoE (Qwen3-MoE experts). The reference runs dense experts through
 * FusedMoe.forward, srt/model_executor/layers/fused_moe/fused.py:205-233;
 * these entry points give the same pipeline over AWQ expert weights.
 */
/* softmax over E router logits (fp32) and top-k; renormalize divides by the
 * top-k sum and then by (sum + 1e-8). Replaces fused_topk, fused.py:11-31. */
int awqb_moe_topk_softmax(const float* logits, int64_t M, int64_t E, int64_t topk,
                          int renormalize, float* topk_weights, int32_t* topk_ids, void* stream);
/* Length of sorted_ids needed by awqb_moe_align. */
int64_t awqb_moe_max_padded(int64_t numel, int64_t num_experts, int64_t block_m);
/* Sort the numel = M*topk (token, k) pairs routed to experts [e_begin, e_end)
 * by expert (stable), pad each expert to block_m with the sentinel numel, write
 * the local expert index of every block and the padded row count.
 * Replaces moe_align_block_size, fused.py:34-61. */
int awqb_moe_align(const int32_t* topk_ids, int64_t numel, int64_t e_begin, int64_t e_end,
                   int64_t block_m, int32_t* sorted_ids, int64_t max_padded,
                   int32_t* block_expert, int32_t* num_post_pad, void* stream);
/* The same result computed by many CTAs (chunk histograms, one scan CTA, one
 * warp per chunk for the stable scatter): for large inputs (thousands of pairs),
 * where one CTA is bound by a single SM. Needs a caller-owned workspace of
 * awqb_moe_align_workspace_bytes(numel, e_end - e_begin) bytes (per-chunk
 * counts; no zeroing needed). Replaces moe_align_block_size, fused.py:34-61. */
int64_t awqb_moe_align_workspace_bytes(int64_t numel, int64_t num_experts);
int awqb_moe_align_ex(const int32_t* topk_ids, int64_t numel, int64_t e_begin, int64_t e_end,
                      int64_t block_m, int32_t* sorted_ids, int64_t max_padded, int32_t* block_expert,
                      int32_t* num_post_pad, void* workspace, int64_t workspace_bytes, void* stream);
/* out[r] = x[sorted_ids[r] / topk] (zero for padding rows), r < *num_post_pad.
 * Stands in for the row gather done by fused_moe_kernel's a_ptrs,
 * kernels/triton/fused_moe.py:241. */
int awqb_moe_gather_rows(const void* x, int64_t K, const int32_t* sorted_ids,
                         const int32_t* num_post_pad, int64_t numel, int64_t topk,
                         int64_t rows_max, void* out, void* stream);
/* Grouped W4A16 GEMM over expert-sorted rows: blobs holds one blob per expert,
 * blob_stride bytes apart (awqb_repack with batch = E). ntok must equal the
 * align block size. Optional row_map / row_scale scatter rows to
 * row_map[r] (< num_valid) and multiply by row_scale[that row].
 * Replaces fused_moe_kernel, kernels/triton/fused_moe.py:155-285. */
int awqb_moe_grouped_workspace_bytes(int64_t rows_max, int64_t K, int64_t N, int64_t G, int ntok,
                                     int64_t* bytes);
int awqb_moe_grouped_gemm(const void* x_sorted, int64_t rows_max, int64_t K, int64_t N, int64_t G,
                          int dtype, const void* blobs, int64_t blob_stride,
                          const int32_t* block_expert, const int32_t* num_post_pad, int ntok,
                          const int32_t* row_map, const float* row_scale, int64_t num_valid,
                          void* y, int64_t ldy, void* workspace, int64_t workspace_bytes,
                          void* stream);
/* The gate_up projection fused with SiLU-and-mul: y[M][N/2] = silu(x W_gate) *
 * (x W_up), computed from the fp32 accumulators (one rounding). The blob must
 * come from AWQ tensors whose columns are interleaved one by one (column 2j =
 * gate j, column 2j + 1 = up j; ops.interleave_gate_up repacks the AWQ
 * tensors). N % 16 == 0; bias (if any) is interleaved the same way. Replaces the gate_up GEMM + SiluAndMul pair of the MLP
 * (layers/activation.py:11-22, blocks.py:53-57) and of the MoE experts
 * (fused.py:160-178). Workspace as for awqb_gemm. */
int awqb_gemm_silu_mul(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                       const void* blob, const void* bias, void* y, void* workspace,
                       int64_t workspace_bytes, void* stream);
/* The same for the MoE expert gate_up GEMM over expert-sorted rows: y [rows][ldy]
 * with ldy >= N / 2, rows in sorted order (as awqb_moe_grouped_gemm without
 * row_map / row_scale). */
int awqb_moe_grouped_gemm_silu_mul(const void* x_sorted, int64_t rows_max, int64_t K, int64_t N,
                                   int64_t G, int dtype, const void* blobs, int64_t blob_stride,
                                   const int32_t* block_expert, const int32_t* num_post_pad, int ntok,
                                   void* y, int64_t ldy, void* workspace, int64_t workspace_bytes,
                                   void* stream);
/* out[r][j] = silu(in[r][j]) * in[r][I + j] in fp32; rows = min(rows_max,
 * *rows_dev) when rows_dev is given. Replaces silu_and_mul (flashinfer),
 * srt/model_executor/layers/activation.py:11-15. */
int awqb_silu_and_mul(const void* in, int64_t rows_max, const int32_t* rows_dev, int64_t I,
                      int dtype, void* out, void* stream);
/* The same for gate_up outputs in the interleaved layout of awqb_gemm_silu_mul
 * (in[r][2j] = gate j, in[r][2j + 1] = up j). */
int awqb_silu_and_mul_interleaved(const void* in, int64_t rows_max, const int32_t* rows_dev, int64_t I,
                                  int dtype, void* out, void* stream);
/* out[m][h] = sum_k in[m][k][h] (fp32 accumulate), counting only pairs whose
 * expert is in [e_begin, e_end) when topk_ids is given.
 * Replaces moe_sum_reduce_triton, kernels/moe_triton.py:68-102. */
int awqb_moe_topk_sum(const void* in, int64_t M, int64_t topk, int64_t H, const int32_t* topk_ids,
                      int64_t e_begin, int64_t e_end, int dtype, void* out, void* stream);

/* ------------------------------------------------------------------------
 * RMSNorm after a projection. Replace flashinfer.rmsnorm and
 * flashinfer.fused_add_rmsnorm as called by RMSNorm / RMSNormFused,
 * srt/model_executor/layers/norm.py:10-47 (arithmetic of flashinfer 0.6.11,
 * include/flashinfer/norm.cuh): per row, x = input (+ residual) in fp32,
 * out = x * rsqrt(mean(x * x) + eps) * weight, rounded to the dtype.
 * N (features) is a multiple of 8 and at most 16384; row strides ld_* are in
 * elements, multiples of 8; all pointers 16-byte aligned. The kernels are
 * launched with programmatic dependent launch after a GEMM on the same stream.
 * ------------------------------------------------------------------------ */
/* out[m] = RMSNorm(input[m]) * weight (out may equal input). */
int awqb_rmsnorm(const void* input, const void* weight, void* out, int64_t M, int64_t N, int64_t ld_in,
                 int64_t ld_out, float eps, int dtype, void* stream);
/* In place: residual[m] = input[m] + residual[m] (rounded), then
 * input[m] = RMSNorm(fp32 sum) * weight. */
int awqb_fused_add_rmsnorm(void* input, void* residual, const void* weight, int64_t M, int64_t N,
                           int64_t ld_in, int64_t ld_res, float eps, int dtype, void* stream);

/* ------------------------------------------------------------------------
 * Tensor-parallel all-reduce. Replaces NCCLWrapper (create_nccl_uid, ctor,
 * all_reduce), kernels/csrc/src/pynccl.cu:75-189, used through
 * PyNCCLDistributedImpl.all_reduce, srt/distributed/communicator.py:62-65.
 * sym_bytes > 0 allocates an ncclMemAlloc buffer registered as a symmetric
 * window (the reference's max_bytes buffer); reductions up to that size are
 * staged through it. awqb_nccl_init allocates (NCCL-owned) memory.
 */
int awqb_nccl_unique_id_bytes(void);
int awqb_nccl_get_unique_id(uint8_t* out);
int awqb_nccl_init(const uint8_t* uid, int rank, int world, int64_t sym_bytes, void** comm);
int awqb_nccl_symmetric_buffer(void* comm, void** ptr, int64_t* bytes);
int awqb_nccl_all_reduce(void* comm, void* buf, int64_t count, int dtype, void* stream);
int awqb_nccl_destroy(void* comm);

/* ------------------------------------------------------------------------
 * Row-parallel GEMM fused with its all-reduce over peer memory (NVLink).
 * Replaces, for small M, the pair RowParallelLinear.forward
 * (layers/linear.py:189-194) = quantised GEMM + PyNCCLCommunicator.all_reduce
 * (kernels/csrc/src/pynccl.cu:96-138): every rank computes its K-slice
 * product and writes each finished value, as one 8-byte {fp32, call tag} word,
 * into every rank's landing buffer; each rank waits for the world words of its
 * values (no fences or flags: the tag travels with the value), sums them in
 * rank order (identical bits on all ranks), adds the bias once and stores
 * y [M][N] in the activation dtype. One kernel, no NCCL call.
 *
 * Set-up, once per rank of the group (collective in spirit: every rank must do
 * it): awqb_tp_exchange_create allocates this rank's exchange buffer
 * (cudaMalloc, (16 * world + 8) * max_rows * max_n bytes + 256) on the current
 * device; exchange the awqb_tp_exchange_handle bytes of all ranks (any host
 * channel), then awqb_tp_exchange_open(ctx, handles of ranks 0..world-1 back to
 * back). Every rank must then issue the same sequence of awqb_gemm_allreduce
 * calls with the same M, K, N, G (a collective); M <= max_rows, N <= max_n.
 * The kernel waits (bounded, 2 s) for its peers' tiles: a rank that does not
 * take part turns into a device error (awqb_device_error), not a hang. The
 * context may be used inside CUDA graphs (no host state changes per call).
 */
int awqb_tp_exchange_handle_bytes(int64_t* bytes);
int awqb_tp_exchange_create(int rank, int world, int64_t max_rows, int64_t max_n, void** ctx);
int awqb_tp_exchange_handle(void* ctx, void* handle_out);
int awqb_tp_exchange_open(void* ctx, const void* handles);
/* Exchange pattern of the fused all-reduce (every rank must set the same):
 * 0 auto (reduce-scatter + all-gather from 4 ranks and 8 rows, on launches
 * that split K over a thread-block cluster; all-to-all otherwise), 1 always
 * all-to-all (each rank sends its partial to every rank; every rank sums),
 * 2 reduce-scatter + all-gather wherever the launch allows it (each rank sends
 * its partial of feature tile t to rank t % world only; that rank sums and
 * sends the rounded result to the others). Results are bit-identical across
 * modes: every sum is taken in rank order. No counterpart in the reference. */
int awqb_tp_exchange_set_mode(void* ctx, int mode);
int awqb_tp_exchange_destroy(void* ctx);
int awqb_gemm_allreduce(const void* x, int64_t M, int64_t K, int64_t N, int64_t G, int dtype,
                        const void* blob, const void* bias, void* y, void* workspace,
                        int64_t workspace_bytes, void* ctx, void* stream);

/* Device-side error word (bits set when a bounded wait inside a kernel gave
 * up). Both calls synchronise the current device. */
int awqb_device_error(uint32_t* out);
int awqb_clear_device_error(void);

#ifdef __cplusplus
}
#endif

#endif /* AWQB200_H */
