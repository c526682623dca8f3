/*
 * mtgemm.h -- C ABI of libmtgemm.so, the B200 (sm_100a) engine for miniTensor's fp32
 * dense-contraction path: matmul / bmm / Linear / Conv2D-as-GEMM.
 *
 * The reference (dionkadi/miniTensor) reaches its GPU kernels through C++ templates
 * declared in include/TensorOps.hpp:697-728 and defined in src/gpu_ops.cpp. Each
 * mt_*_gpu function below replaces one of them for T = float, with the same argument
 * meaning, so a binding only maps a Tensor<float> to an mt_tensor (storage pointer,
 * view offset, shape, strides -- exactly the fields of include/TensorImpl.hpp) and
 * turns a non-zero status into the reference's exception (std::runtime_error carrying
 * mt_last_error()).
 *
 * Conventions (the reference's, include/TensorOps.hpp:993-1149, include/GpuUtils.hpp):
 *   - All pointers are device pointers (except the A, B and C of mt_matmul_host, which are
 *     host buffers). The caller allocates every output with its final shape; the callee
 *     overwrites it (gradient accumulation stays with the caller).
 *   - Inputs are borrowed views: data + offset is element (0,...,0); strides are in
 *     elements; stride 0 marks a broadcast (expand) dimension. Unlike the reference's
 *     matmul_gpu (src/gpu_ops.cpp:1125-1127), view offsets are always honoured.
 *   - Launches are asynchronous on `stream` (NULL = legacy default stream, the
 *     reference's active_stream() default); nothing synchronises inside a call, so calls
 *     can be captured in CUDA graphs.
 *   - Device memory: four paths take stream-ordered scratch (cudaMallocAsync and
 *     cudaFreeAsync on `stream`; inside a capture these become graph memory nodes):
 *       . a GEMM whose output has too few tiles to fill the GPU (batch 1, no extra
 *         destinations, at least 8 k-blocks): its k range is split, the fp32 partials go
 *         to a split x M x N array and a second kernel sums them in split order;
 *       . a stride-1 tensor-core conv forward or input gradient: an NHWC copy of the
 *         activation (or of dY) and the weights reordered tap by tap;
 *       . the conv weight gradient, stated below (mt_conv2d_wgrad can take a caller
 *         workspace, mt_conv2d_wgrad_noalloc a fixed library array);
 *       . mt_matmul_host without a workspace: the device copies of A, B and C.
 *     Strict-fp32 calls and every other path allocate nothing.
 *   - Every function returns an mt_status and never throws; mt_last_error() gives the
 *     thread-local message of the last failure.
 */
#ifndef MTGEMM_H
#define MTGEMM_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define MT_API __declspec(dllexport)
#else
#define MT_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define MT_MAX_DIMS 8 /* include/Defines.hpp:8 MAX_DIMS */

/* A strided view, field for field the reference's TensorImpl
 * (include/TensorImpl.hpp:153-160: storage_, shape_, strides_, offset_). */
typedef struct mt_tensor {
    float* data;                   /* storage base = Tensor<float>::data() (include/Tensor.hpp:80) */
    uint64_t offset;               /* Tensor::offset(), elements */
    uint32_t ndim;                 /* <= MT_MAX_DIMS */
    uint64_t shape[MT_MAX_DIMS];
    uint64_t strides[MT_MAX_DIMS]; /* elements; 0 = broadcast */
} mt_tensor;

typedef enum mt_status {
    MT_OK = 0,
    MT_EINVAL = 1,        /* shape/argument error (reference: std::invalid_argument) */
    MT_EUNSUPPORTED = 2,  /* valid request this build does not serve */
    MT_ECUDA = 3,         /* CUDA runtime error (reference: GPU_CHECK -> std::runtime_error) */
    MT_ETIMEOUT = 4,      /* a device-side bounded wait gave up (mt_device_status) */
    MT_ENOMEM = 5
} mt_status;

/* Arithmetic of the fp32-input contraction. */
typedef enum mt_mode {
    MT_MODE_DEFAULT = -1, /* process default: env MT_GEMM_MODE (strict|tf32|tf32x3), else TF32X3 */
    MT_STRICT_FP32 = 0,   /* FFMA only (SIMT kernel), k ascending per output */
    MT_TF32 = 1,          /* tcgen05 kind::tf32, one MMA per k-step */
    MT_TF32X3 = 2         /* tcgen05 split precision hi*hi + hi*lo + lo*hi (fp32-accurate) */
} mt_mode;

/* Fused epilogue flags (applied after the full k-sum, in this order). */
enum {
    MT_EPI_NONE = 0,
    MT_EPI_BIAS_ROW = 1, /* C[m,n] += bias[m] */
    MT_EPI_BIAS_COL = 2, /* C[m,n] += bias[n]   (Linear: bias [1,out]) */
    MT_EPI_RELU = 4      /* C = max(C, 0) */
};

/* ---- mirrors of the reference GPU entry points (T = float) -------------------------- */

/* include/TensorOps.hpp:703 matmul_gpu(A, B, C): C[M,N] = A[M,K] * B[K,N].
 * Called by matmul() (include/TensorOps.hpp:1026) for contiguous operands. */
MT_API int mt_matmul_gpu(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream);

/* include/TensorOps.hpp:704 matmul_gpu_strided: same contract, arbitrary 2-D strides
 * (the transposed views of MatmulBackward, include/Autograd.hpp:131-141). */
MT_API int mt_matmul_gpu_strided(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream);

/* include/TensorOps.hpp:705 matmul_gpu_v2 and :706 matmul_gpu_bk16 (benchmark names of
 * the same GEMM, src/gpu_ops.cpp:1167-1197). */
MT_API int mt_matmul_gpu_v2(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream);
MT_API int mt_matmul_gpu_bk16(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream);

/* Replaces the per-batch loop of bmm() (include/TensorOps.hpp:933-991, which makes both
 * operands contiguous and launches one matmul_gpu per batch): one launch over
 * C[b,M,N] = A[b,M,K] * B[b,K,N]; a batch stride of 0 (expand) is read in place. */
MT_API int mt_bmm_gpu(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, void* stream);

/* Linear<float>::forward (include/Module.hpp:112-114: matmul(x, W) + bias) as one GEMM
 * with the bias add (and optional ReLU) fused into the epilogue. X [M,in], W [in,out]
 * (the reference's layout), bias [1,out] or [out] or NULL, Y [M,out]. */
MT_API int mt_linear_fwd_gpu(const mt_tensor* X, const mt_tensor* W, const mt_tensor* bias,
                             const mt_tensor* Y, int relu, void* stream);

/* ---- Conv2D (NCHW) as implicit GEMM --------------------------------------------------
 * x [N,C,H,W], w [C_out,C,kh,kw], y / dY [N,C_out,H_out,W_out] with
 * H_out = (H + 2*padding - kh) / stride + 1 (0 when H + 2*padding < kh), as
 * safe_out_size (include/TensorOps.hpp:17-20). Inputs may be strided views; outputs must be
 * contiguous (as the reference allocates them). */

/* include/TensorOps.hpp:708 conv2d_gpu(input, weight, bias, output, stride, padding);
 * bias may be NULL or empty. Called by conv2d() (include/TensorOps.hpp:1096). */
MT_API int mt_conv2d_gpu(const mt_tensor* in, const mt_tensor* w, const mt_tensor* bias, const mt_tensor* out,
                         uint64_t stride, uint64_t padding, void* stream);

/* include/TensorOps.hpp:709 conv2d_gpu_strided: same contract for non-contiguous inputs
 * (the reference's conv2d() picks it when a view is not contiguous, :1097). */
MT_API int mt_conv2d_gpu_strided(const mt_tensor* in, const mt_tensor* w, const mt_tensor* bias,
                                 const mt_tensor* out, uint64_t stride, uint64_t padding, void* stream);

/* include/TensorOps.hpp:710 conv2d_backward_input_gpu(grad_output, weight, grad_input, ...). */
MT_API int mt_conv2d_backward_input_gpu(const mt_tensor* dY, const mt_tensor* w, const mt_tensor* dX,
                                        uint64_t stride, uint64_t padding, void* stream);

/* include/TensorOps.hpp:711 conv2d_backward_weight_gpu(grad_output, input, grad_weight, ...).
 * The tensor-core path splits the reduction over output pixels; its fp32 partials live in a
 * stream-ordered allocation (cudaMallocAsync on `stream`, freed on the same stream), summed
 * in a fixed order. mt_conv2d_wgrad takes a caller workspace instead. */
MT_API int mt_conv2d_backward_weight_gpu(const mt_tensor* dY, const mt_tensor* x, const mt_tensor* dW,
                                         uint64_t stride, uint64_t padding, void* stream);

/* include/TensorOps.hpp:712 conv2d_backward_bias_gpu(grad_output, grad_bias): db[co] is the
 * sum over n (ascending) of the spatial sum of dY[n,co], the order of :398-418. */
MT_API int mt_conv2d_backward_bias_gpu(const mt_tensor* dY, const mt_tensor* db, void* stream);

/* out[n] = sum over m of X[m, n] for a 2-D view X [M, N] and a 1-D (or [1, N]) view out:
 * the axis-0 sum that unbroadcast (include/TensorOps.hpp:1305-1345) applies to the bias
 * gradient of Linear (forward = matmul(x, W) + bias, include/Module.hpp:112-114). The
 * reference runs it through its own reduction kernels; this is not one of its nine GPU
 * entry points. Order: 8 partial sums over rows m = w (mod 8), each ascending, then added
 * in order w = 0..7 (deterministic). */
MT_API int mt_sum_rows_gpu(const mt_tensor* X, const mt_tensor* out, void* stream);

/* Explicit-mode variants of the three convolution products. */
MT_API int mt_conv2d_fwd(const mt_tensor* x, const mt_tensor* w, const mt_tensor* bias, const mt_tensor* y,
                         uint64_t stride, uint64_t padding, int mode, void* stream);
MT_API int mt_conv2d_dgrad(const mt_tensor* dy, const mt_tensor* w, const mt_tensor* dx, uint64_t stride,
                           uint64_t padding, int mode, void* stream);
/* workspace == NULL: stream-ordered allocation as above; else at least
 * mt_conv2d_wgrad_workspace_bytes(...) bytes of device memory, used only by this call. */
MT_API int mt_conv2d_wgrad(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw, uint64_t stride,
                           uint64_t padding, int mode, void* workspace, size_t ws_bytes, void* stream);
/* Workspace size for mt_conv2d_wgrad (0: none needed or invalid shapes); reads only the
 * shapes of its arguments, so their data pointers may be NULL. */
MT_API size_t mt_conv2d_wgrad_workspace_bytes(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw,
                                              uint64_t stride, uint64_t padding, int mode);

/* Channels-last copy of an (N, C, H, W) view: out has x's shape with strides
 * (H*W*C, 1, W*C, C), C a multiple of 4, start 16-byte aligned; x and out must not overlap.
 * No counterpart in the reference, which keeps every tensor NCHW. The stride-1 tensor-core
 * convolutions work on NHWC and transform an NCHW input on every call; given such a copy
 * (for x, or dy in mt_conv2d_dgrad) they read it in place. A training step whose forward
 * and weight gradient share one input therefore transforms it once: mt_conv2d_fwd and
 * mt_conv2d_wgrad on the same copy (the path string ends in " nhwc_in"). Results are
 * bitwise those of the NCHW input. */
MT_API int mt_nchw_to_nhwc(const mt_tensor* x, const mt_tensor* out, void* stream);

/* Weight gradient that allocates nothing: no counterpart in the reference. For callers
 * that cannot allocate device memory during the call (a graph capture that forbids
 * allocation nodes, a host that owns all device memory, a latency-critical loop). It
 * computes what mt_conv2d_wgrad computes, with the split-K partials in a fixed 8 MiB
 * array inside the library (one per GPU, held until the process exits); problems whose
 * partials need more get MT_EINVAL with the size in the message. The first call on a
 * device looks up that array's device address, so make it before any stream capture
 * (after a device reset, the first call looks it up again). It always takes the gather
 * kernel, whose only scratch is those partials. All calls on a device share the array:
 * calls that overlap on the GPU (other streams, other host threads) race and must be
 * serialised by the caller. */
MT_API int mt_conv2d_wgrad_noalloc(const mt_tensor* dy, const mt_tensor* x, const mt_tensor* dw, uint64_t stride,
                                   uint64_t padding, int mode, void* stream);

/* ---- general entry point ----------------------------------------------------------- */

/* C = epi(A * B) for 2-D or 3-D (batched) views with an explicit mode. `bias` is a device
 * pointer of M (BIAS_ROW) or N (BIAS_COL) floats, shared by all batches. */
MT_API int mt_gemm(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C,
                   const float* bias, int epi, int mode, void* stream);

/* C[M,N] = A[M,K] * B[K,N] for row-major HOST buffers. Replaces the reference's sequence for
 * host data: A.to(cuda), B.to(cuda), matmul(), C.to(cpu). There, each to() is a synchronous
 * cudaMemcpy of the whole storage (include/TensorImpl.hpp:245-275) and matmul() runs in
 * between (include/TensorOps.hpp:993-1045). Here the three overlap. B goes to the device
 * first, then A in `panels` row panels on a library copy stream. The GEMM of panel i starts
 * on `stream` once its rows have landed, and C's panel i returns on a second copy stream
 * while later panels still arrive. The PCIe directions are independent, so the step costs
 * about the host-to-device transfer plus one panel.
 *   - Host buffers should be pinned (cudaHostAlloc / cudaHostRegister) for the copies to
 *     overlap; pageable buffers work, serialised. They must stay valid, and C unread,
 *     until `stream` has completed: the call only queues the work.
 *   - `workspace` (device, 256-byte aligned, >= mt_matmul_host_workspace_bytes) holds A, B
 *     and C on the device; NULL takes a stream-ordered allocation on `stream`.
 *   - panels <= 0 picks the default (8, fewer for short A); panels are whole 256-row tiles.
 *   - The two copy streams are per device and shared by all calls on that device. */
MT_API int mt_matmul_host(const float* A, const float* B, float* C, uint64_t M, uint64_t K, uint64_t N,
                          int mode, int panels, void* workspace, size_t ws_bytes, void* stream);
MT_API size_t mt_matmul_host_workspace_bytes(uint64_t M, uint64_t K, uint64_t N);

/* ---- multi-GPU: a column-sharded GEMM whose epilogue all-gathers C ------------------
 * The reference is single-GPU (README.md:273); these entry points have no counterpart
 * there. One process per GPU: rank r holds A and the column shard B[:, n0:n1], computes
 * C[:, n0:n1] and its epilogue stores every tile into its own C and into each peer's C
 * (CUDA IPC peer pointers over NVLink), then mt_peer_barrier makes the writes visible. */

/* IPC handle (64 bytes) of the allocation containing dptr, plus dptr's byte offset in it. */
MT_API int mt_ipc_get_handle(const void* dptr, void* handle_out, uint64_t* offset_out);
/* Maps a peer's handle into this process; *dptr_out = mapped base + offset. */
MT_API int mt_ipc_open(const void* handle, uint64_t offset, void** dptr_out);
MT_API int mt_ipc_close(void* dptr, uint64_t offset);

/* C = epi(A * B) written to C and to extra_dst[0..nextra) (nextra < 8), each a device
 * pointer (peer-mapped allowed) laid out with C's row (and batch) strides. A, B and C are
 * 2-D, or 3-D with a common batch (batch stride 0 = an operand broadcast over the batch):
 * a batch-sharded bmm passes its block of batches, and the epilogue writes every finished
 * tile to every rank's C. */
MT_API int mt_gemm_multi(const mt_tensor* A, const mt_tensor* B, const mt_tensor* C, float* const* extra_dst,
                         int nextra, const float* bias, int epi, int mode, void* stream);

/* Stream-ordered cross-GPU barrier: flags[d] is rank d's array of `world` ints (peer-mapped,
 * zero-initialised). Rank `rank` stores `epoch` into flags[d][rank] for every d, then waits
 * until flags[rank][*] == epoch. The wait gives up after timeout_ns and records status 6 in
 * the device status word (mt_device_status) instead of hanging. timeout_ns above 60 s
 * (60e9) is refused with MT_EINVAL, so that every device-side wait stays bounded. */
MT_API int mt_peer_barrier(int* const* flags, int rank, int world, int epoch, uint64_t timeout_ns, void* stream);

/* Stream-ordered 2-D copy of `rows` rows of `width_bytes` bytes (row pitches dpitch /
 * spitch bytes) from src to dst, by the copy engines -- dst may be a peer-mapped pointer,
 * which makes this a push over NVLink without SM involvement. One cudaMemcpy2DAsync. */
MT_API int mt_copy_rows_async(void* dst, uint64_t dpitch, const void* src, uint64_t spitch, uint64_t width_bytes,
                              uint64_t rows, void* stream);

/* ---- scratch memory ------------------------------------------------------------------ */

/* Where the library's temporary device buffers come from (split-K and stream-K partials,
 * the stride-1 conv's NHWC copy and reordered weights, weight-grad partials). The
 * reference takes scratch from its MemoryPool (include/MemoryPool.hpp:45-99); its drop-in
 * overlay installs the pool here. With no allocator installed (the default, or after
 * passing NULL, NULL) every buffer is a stream-ordered allocation on the call's stream from
 * the library's own per-device pool (cudaMallocFromPoolAsync / cudaFreeAsync; the pool
 * keeps freed memory cached for the next call). With one installed, alloc(bytes, device, ctx) is called before the
 * kernels are enqueued and free(ptr, bytes, device, ctx) right after: the block may be
 * handed out again while those kernels still run, so work sharing the allocator must be
 * ordered on one stream (the reference's active_stream()). A NULL from alloc fails the
 * call with MT_ENOMEM. Install it once, before other calls; mt_matmul_host keeps its
 * stream-ordered workspace (it spans several streams) unless given one. */
typedef void* (*mt_scratch_alloc_fn)(size_t bytes, int device, void* ctx);
typedef void (*mt_scratch_free_fn)(void* ptr, size_t bytes, int device, void* ctx);
MT_API int mt_set_scratch_allocator(mt_scratch_alloc_fn alloc, mt_scratch_free_fn free_fn, void* ctx);
/* Scratch buffers obtained so far (all threads): stream-ordered, and from the installed
 * allocator. */
MT_API void mt_scratch_counts(uint64_t* stream_ordered, uint64_t* from_allocator);

/* ---- process settings and diagnostics ---------------------------------------------- */

MT_API int mt_set_default_mode(int mode);   /* returns the previous default */
MT_API int mt_get_default_mode(void);
MT_API const char* mt_last_error(void);     /* thread-local */
/* Kernel chosen by this thread's last successful call, e.g. "umma_tf32x3 bn=256 a=K b=MN". */
MT_API const char* mt_last_path(void);
/* Kernels launched by this library since load (all threads). */
MT_API uint64_t mt_launch_count(void);
/* Synchronises the current device and returns its device status word (0 = clean,
 * else the code of the first bounded wait that gave up); reset != 0 clears it. */
MT_API int mt_device_status(int reset);
/* Library version string. */
MT_API const char* mt_version(void);

#ifdef __cplusplus
}
#endif
#endif /* MTGEMM_H */
