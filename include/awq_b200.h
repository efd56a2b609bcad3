/*
 * awq_b200.h -- C ABI of the B200 (sm_100a) AWQ W4A16 library, libawq_b200.so.
 *
 * Drop-in boundary for songqiuyu/Qwen2-7B-Triton_Engine's AWQ matrix product.
 * Every entry point takes plain pointers and sizes; device pointers are owned by
 * the caller and never freed here.  Streams are passed as `void*` holding a
 * cudaStream_t (NULL = the legacy default stream).  The product entry points
 * allocate no device memory and never synchronize: they only enqueue kernels on
 * `stream`.  The exceptions are named where they are declared: the
 * tensor-parallel set-up and tear-down (awq_tp_comm_create / _create_ex / _open /
 * _destroy) allocate, map or free a buffer and synchronize the device, awq_tp_comm_reset
 * synchronizes the device, and
 * awq_device_status synchronizes `stream`.  Nothing throws; each entry point
 * returns AWQ_OK (0) or a negative AWQ_ERR_* code, and awq_last_error() gives a
 * message for the calling thread.
 *
 * Packed layout (model/qwen2.py:34-36, kernels/awq_gemm.py:36-38):
 *   qweight int32 [K, N/8]   row-major; element n of row k is the nibble at bit
 *                            4 * order[n % 8] of word n / 8, order = 0,4,1,5,2,6,3,7
 *   qzeros  int32 [K/gs, N/8]
 *   scales  fp16  [K/gs, N]
 *   W[k, n] = fp16(w - z) * scale in fp16 (kernels/awq_gemm.py:59)
 * Requirements: N % 8 == 0, group_size % 8 == 0, K % group_size == 0; qweight,
 * qzeros, scales and out 16-byte aligned and densely packed (row stride = width);
 * x rows of length K with stride ldx >= K (elements), 2-byte aligned.
 */
#ifndef AWQ_B200_H_
#define AWQ_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AWQ_API __attribute__((visibility("default")))
#else
#define AWQ_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define AWQ_OK 0
#define AWQ_ERR_INVALID_ARG (-1)   /* null pointer, bad shape, bad alignment       */
#define AWQ_ERR_UNSUPPORTED (-2)   /* valid input this build cannot run (e.g. path) */
#define AWQ_ERR_CUDA (-3)          /* a CUDA runtime call failed                    */
#define AWQ_ERR_WORKSPACE (-4)     /* workspace missing or too small                */
#define AWQ_ERR_DEVICE (-5)        /* a kernel reported an error (awq_device_status) */

/* Kernel choice for awq_gemm_f16_ex. */
#define AWQ_PATH_AUTO 0   /* M <= 8: decode kernel; 9..16: small-M tcgen05 kernel (AWQ_PATH_TS)
                             when the shape allows, else decode; larger M: tcgen05 GEMM when
                             the shape allows and its CTAs (output tiles x K splits, the
                             splits needing the workspace) fill at least half the SMs or
                             M > 64, else decode                                            */
#define AWQ_PATH_DECODE 1 /* mma.sync split-K streaming kernel, any M (16-token chunks)          */
#define AWQ_PATH_TC 2     /* tcgen05/TMEM prefill GEMM; AWQ_ERR_UNSUPPORTED if shape disallows   */
#define AWQ_PATH_TS 3     /* tcgen05 small-M GEMM (M <= 64): weights dequantized into TMEM as the
                             MMA's A operand, tokens as its N; AWQ_ERR_UNSUPPORTED otherwise    */

/* Library version: major * 10000 + minor * 100 + patch. */
AWQ_API int awq_version(void);

/* Message describing the last error returned on this thread ("" if none). */
AWQ_API const char* awq_last_error(void);

/*
 * Bit-exact dequantization: out fp16 [K, N] = W.
 * Replaces _dequant_to_fp16 / _dequant_awq_kernel (kernels/awq_gemm.py:14-87).
 */
AWQ_API int awq_dequant_f16(const int32_t* qweight, const int32_t* qzeros, const void* scales, void* out,
                    int64_t K, int64_t N, int64_t group_size, void* stream);

/*
 * Bytes of workspace awq_gemm_f16 / awq_gemm_f16_ex need for this shape on the
 * current device (0 is a valid answer).  The workspace holds split-K partial sums
 * and arrival counters.  It must be zero-filled once before its first use
 * (awq_workspace_init); every completed call leaves the counters at zero again.
 * Calls that run concurrently (different streams) need different workspaces.
 * No counterpart in the reference (its M<=4 path keeps a global K*N fp16 buffer,
 * kernels/awq_gemm.py:234,255-262).
 */
AWQ_API size_t awq_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int64_t group_size);

/* Zero-fill a workspace on `stream` (cudaMemsetAsync). */
AWQ_API int awq_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/*
 * out fp16 [M, N] (row stride ldo) = x fp16 [M, K] (row stride ldx) @ W, fp32
 * accumulation.  Replaces awq_gemm_forward (kernels/awq_gemm.py:237-284) after its
 * reshape of x to [M, K]: M <= 8 runs the decode kernel, 9 <= M <= 16 the small-M
 * tcgen05 kernel, larger M the tcgen05 prefill GEMM, each when the shape allows it,
 * else the decode kernel over 16-token chunks (AWQ_PATH_AUTO below).
 */
AWQ_API int awq_gemm_f16(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                 const void* scales, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                 int64_t group_size, void* workspace, size_t workspace_bytes, void* stream);

/* awq_gemm_f16 with an explicit kernel choice (AWQ_PATH_*), for tests and benchmarks. */
AWQ_API int awq_gemm_f16_ex(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                    const void* scales, void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                    int64_t group_size, void* workspace, size_t workspace_bytes, void* stream,
                    int path);

/*
 * out = x @ W + bias: the product with the bias of the layer added in its epilogue
 * (bias fp16 [N], added to every row in fp32 before the one fp16 rounding).  Replaces
 * the awq_gemm_forward + `out + bias` pair of the reference's biased linears
 * (model/qwen2.py:45-46 for LinearAWQ, :108-109 for the fused q/k/v), saving the second
 * kernel and a write and read of the output.  Same kernels and requirements as
 * awq_gemm_f16 (AWQ_PATH_AUTO).
 */
AWQ_API int awq_gemm_f16_bias(const void* x, int64_t ldx, const int32_t* qweight,
                              const int32_t* qzeros, const void* scales, const void* bias,
                              void* out, int64_t ldo, int64_t M, int64_t N, int64_t K,
                              int64_t group_size, void* workspace, size_t workspace_bytes,
                              void* stream);

/*
 * out = silu(G) * U for the fused gate+up product P = x @ W (W = [gate | up], N
 * columns): G = P[:, :N/2], U = P[:, N/2:], out fp16 [M, N/2] (ldo >= N/2).  Replaces the
 * reference MLP's awq_gemm_forward + two .contiguous() slices + silu_mul_forward
 * (model/qwen2.py:181-194, kernels/silu_mul.py:41-64): fp16-rounded G and U, fp32
 * x * sigmoid(x) * y, one fp16 rounding.  Up to 8 tokens with N/2 a multiple of 256 the
 * decode kernel pairs each gate strip with its up strip in its epilogue (P is never
 * written); from 9 tokens up, with N a multiple of 512 and enough output tiles to run
 * without a K split, the tcgen05 kernels do the same in theirs; otherwise the product
 * goes to a temporary inside the workspace and one elementwise kernel follows.  Workspace: awq_gemm_silu_mul_workspace_bytes bytes,
 * zero-filled once (awq_workspace_init), the same buffer the other calls use.
 */
AWQ_API size_t awq_gemm_silu_mul_workspace_bytes(int64_t M, int64_t N, int64_t K,
                                                 int64_t group_size);
AWQ_API int awq_gemm_f16_silu_mul(const void* x, int64_t ldx, const int32_t* qweight,
                                  const int32_t* qzeros, const void* scales, void* out,
                                  int64_t ldo, int64_t M, int64_t N, int64_t K,
                                  int64_t group_size, void* workspace, size_t workspace_bytes,
                                  void* stream);

/*
 * awq_gemm_f16 for callers that cannot allocate device memory: same inputs and
 * output, no workspace argument.  This entry point has no counterpart in the
 * reference.  It serves hosts that forbid allocation on the path where the product
 * runs -- an engine that plans all device memory up front (cudaMalloc / cudaFree can
 * synchronize the device and stall every stream), or a plugin interface that hands
 * the library only its input and output buffers.
 *   - Runs the generic decode kernel (any M, 16-row chunks; fastest for M <= 16).
 *   - Its split-K scratch is a 4 MiB file-scope device array, held by every GPU that
 *     loads the library until the process exits.  The split factor is reduced until the
 *     partial sums fit; a shape that still does not fit returns AWQ_ERR_WORKSPACE.
 *   - The first call on a device looks up the array's device address (with that
 *     device current): make that first call before any stream capture.  The array's
 *     counters start at zero because a device array is zero-initialised when the
 *     library's module loads, and every call leaves them at zero again.
 *   - All calls share the array: calls that overlap on the GPU race and give wrong
 *     results.  No allocation of any kind happens inside.
 */
AWQ_API int awq_gemm_f16_noalloc(const void* x, int64_t ldx, const int32_t* qweight,
                                 const int32_t* qzeros, const void* scales, void* out, int64_t ldo,
                                 int64_t M, int64_t N, int64_t K, int64_t group_size, void* stream);

/*
 * The schedule the tcgen05 prefill kernel takes for an M x N x K product on a GPU with
 * num_sms SMs, when the caller's workspace holds what it needs: *kind = AWQ_TC_GRID (one
 * CTA per 256-column output tile, *param = tiles), AWQ_TC_PERSISTENT (more tiles than
 * SMs: one CTA per SM takes tiles in turn, *param = tiles), AWQ_TC_STREAMK (tiles fill
 * half to most of the SMs: *param = K/64 steps each tile's own CTA runs before the other
 * CTAs share the tails) or AWQ_TC_SPLITK (*param = CTAs along K per tile).  Host-only
 * arithmetic: needs no GPU.  No counterpart in the reference (introspection for tests
 * and tuning).
 */
#define AWQ_TC_GRID 0
#define AWQ_TC_PERSISTENT 1
#define AWQ_TC_STREAMK 2
#define AWQ_TC_SPLITK 3
AWQ_API int awq_tc_schedule(int64_t M, int64_t N, int64_t K, int num_sms, int* kind, int* param);

/* 1 if AWQ_PATH_TC can run this shape with these pointers, else 0. */
AWQ_API int awq_tc_supported(const void* x, int64_t ldx, const int32_t* qweight, const int32_t* qzeros,
                     const void* scales, int64_t M, int64_t N, int64_t K, int64_t group_size);

/*
 * Synchronizes `stream`, then reads and clears the current device's kernel status
 * word.  Returns AWQ_OK, or AWQ_ERR_DEVICE with the status bits in *status_out
 * (1 = a bounded barrier wait timed out, 2 = a kernel rejected its parameters,
 * 4 = a fused all-reduce gave up waiting for other ranks).
 * No counterpart in the reference.
 */
AWQ_API int awq_device_status(void* stream, int* status_out);

/*
 * ---- Tensor parallelism: the row-parallel product fused with its all-reduce -------------
 * For the row-parallel linears of a tensor-parallel model (o_proj and down_proj split
 * along K over `world` GPUs of one box, one process per GPU), awq_gemm_f16_allreduce
 * computes this rank's partial product and sums it over all ranks in the same kernel:
 * the CTA that finishes an output tile stores each fp32 value of the tile, packed with
 * the call's flag (the call number + 1) into one 8-byte word, into its slot of every
 * rank's receive buffer over NVLink (CUDA IPC peer mappings, plain stores); it then
 * reads, in its own buffer, every rank's words for the tile until their flags show this
 * call (bounded wait) and sums the values in rank order, so every rank writes the same
 * fp16 bits.  A wait that runs out sets status bit 4 (awq_device_status): the output of
 * that call is then wrong on this rank and the communicator must be reset
 * (awq_tp_comm_reset) on every rank before it is used again.  It replaces the awq_gemm_f16 +
 * NCCL all-reduce pair of a row-parallel layer (the reference has no tensor
 * parallelism: inference/engine.py:15).
 *
 * Set-up, once per rank -- the only entry points that allocate device memory and
 * synchronize the device:
 *   awq_tp_comm_create(world, rank, max_n, handle, &comm)  this rank's buffer + its handle
 *   gather the world handles in rank order (e.g. torch.distributed.all_gather_object)
 *   awq_tp_comm_open(comm, handles)                         maps the other ranks' buffers
 * Every rank must then issue the same sequence of awq_gemm_f16_allreduce calls, in one
 * stream per communicator (CUDA-graph capture is fine).  awq_tp_comm_destroy after the
 * device has finished all calls.  max_n bounds N of the calls (multiple of 8).
 *
 * Above 16 tokens (communicators made by awq_tp_comm_create_ex with max_rows >= M) the
 * product runs on the prefill kernels into an fp16 plane of this rank's buffer, and one
 * all-reduce kernel follows over NVLink: each rank sums its 1/world row slice of every
 * rank's plane in rank order (fp32 accumulation of the fp16 partials, one rounding),
 * stores it into every rank's result plane, and copies the result plane to out once all
 * slices are in -- the same bits on every rank, no NCCL.  Flags carry the call number,
 * as above; the same time-out and reset rules apply.
 */
typedef struct awq_tp_comm awq_tp_comm;
#define AWQ_IPC_HANDLE_BYTES 64
#define AWQ_MAX_WORLD 8

AWQ_API int awq_tp_comm_create(int world, int rank, int64_t max_n, void* handle_out,
                               awq_tp_comm** comm_out);
/* awq_tp_comm_create with room for calls of up to max_rows tokens above 16 (two fp16
 * planes of max_rows x max_n more per rank; max_rows = 0 is awq_tp_comm_create).  No
 * counterpart in the reference. */
AWQ_API int awq_tp_comm_create_ex(int world, int rank, int64_t max_n, int64_t max_rows,
                                  void* handle_out, awq_tp_comm** comm_out);
AWQ_API int awq_tp_comm_open(awq_tp_comm* comm, const void* handles);
/* Longest wait for the other ranks' tiles, in ns (default 2 s); then status bit 4. */
AWQ_API int awq_tp_comm_set_timeout(awq_tp_comm* comm, uint64_t timeout_ns);
/*
 * Return this rank's communicator to its freshly opened state after a wait ran out
 * (status bit 4): synchronizes the device, zeroes this rank's receive buffer and call
 * number, synchronizes again.  A collective step: every rank must call it with no fused
 * call in flight anywhere, between two barriers of the ranks (one before, so that no
 * rank still writes into another's buffer, one after, so that no rank starts a new call
 * before every buffer is clear).  No counterpart in the reference.
 */
AWQ_API int awq_tp_comm_reset(awq_tp_comm* comm);
AWQ_API int awq_tp_comm_destroy(awq_tp_comm* comm);

/* 1 if awq_gemm_f16_allreduce can run this call, else 0 (then use awq_gemm_f16 + an
 * all-reduce).  M <= 16: the decode kernel with one CTA per SM in a single wave (N % 32
 * == 0, group_size % 64 == 0, 16-byte aligned qweight and x, ldx % 8 == 0, N <= max_n).
 * M > 16: M <= the communicator's max_rows and N <= max_n. */
AWQ_API int awq_allreduce_supported(const awq_tp_comm* comm, const void* x, int64_t ldx,
                                    const int32_t* qweight, int64_t M, int64_t N, int64_t K,
                                    int64_t group_size);

/* out[M, N] = sum over ranks of (this rank's x[M, K_r] @ W_r), written on every rank.
 * Workspace as for awq_gemm_f16 (awq_gemm_workspace_bytes). */
AWQ_API int awq_gemm_f16_allreduce(awq_tp_comm* comm, const void* x, int64_t ldx,
                                   const int32_t* qweight, const int32_t* qzeros,
                                   const void* scales, void* out, int64_t ldo, int64_t M,
                                   int64_t N, int64_t K, int64_t group_size, void* workspace,
                                   size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AWQ_B200_H_ */
