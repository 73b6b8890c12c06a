/*
 * mfb.h — C ABI of the B200 (sm_100a) dense FP32 contraction library (libmfb.so).
 *
 * Every entry point takes plain pointers, sizes and a CUDA stream handle; no C++
 * or framework types cross this boundary. All matrices are row-major FP32 with
 * explicit leading dimensions (elements), exactly like the reference's pointer
 * interface. Buffers are caller-owned device memory unless stated otherwise.
 *
 * Replaces (reference file:line):
 *   mfb_cuda_gemm / mfb_cuda_sync   matrix_pro::hw::cuda_gemm / cuda_sync
 *                                   include/matrix_pro/detail/cuda_hooks.hpp:17-18,28
 *                                   (body: src/hw/cuda_backend.cu:91-99,159-163)
 *   mfb_sgemm                       the cublasLtMatmul/cublasGemmEx call of GemmPlan::Impl::run_ptr
 *                                   src/ops/gemm/plan/implementation.inc:128-151
 *   mfb_sgemm_host                  the GPU share of HeterogeneousScheduler::gemm (host operands)
 *                                   src/hw/scheduler.cpp:236-312
 *   mfb_sgemm_strided_batched       cublasSgemmStridedBatched in batch_matmul and its backward
 *                                   src/nn/batch.cu:12-35, src/nn/backward/batched_matmul.inc:7-55
 *   mfb_conv2d_bwd_data / _filter /  conv2d_input_backward / conv2d_weight_backward / conv2d_bias_backward
 *   mfb_conv2d_bwd_bias             include/matrix_pro/nn/conv.hpp:25-29 (kernels:
 *                                   src/nn/backward/convolution_kernels.cuh:9-95)
 *   mfb_all_reduce / _broadcast /    matrix_pro::all_reduce / broadcast / all_gather / reduce_scatter /
 *   _all_gather / _reduce_scatter /  scatter / gather (include/matrix_pro/distributed/collectives.hpp:20-32,
 *   _scatter / _gather              src/hw/collectives.cpp:185-311)
 *   mfb_cuda_nccl_allreduce         hw::cuda_nccl_allreduce (include/matrix_pro/detail/cuda_hooks.hpp:35,
 *                                   stub at src/hw/cuda_backend.cu:252)
 *   mfb_covariance / mfb_correlation matrix_pro::covariance / correlation
 *                                   src/ops/reductions/covariance.inc:23-60
 *   mfb_plan_*                      GemmPlan ctor/execute/tune/rows/cols/inner/candidate_count
 *                                   include/matrix_pro/ops/gemm.hpp:36-62
 *                                   (src/ops/gemm/plan/implementation.inc:5-152, tuning.inc:5-66)
 *   mfb_gemv                        gemm_gemv (gemv_rows_kernel, gemm_skinny_n_kernel, gemv_cols_kernel)
 *                                   src/ops/gemm/gemm_gemv.cu:86-110
 *   mfb_conv2d_fwd                  matrix_pro::conv2d  include/matrix_pro/nn/conv.hpp:16-17
 *                                   (src/nn/conv.cu:110-163)
 *   mfb_naive_sgemm                 the one-thread-per-output comparison GEMM
 *                                   benchmarks/bench_comparison.cu:76 (device correctness oracle)
 */
#ifndef MFB_H_
#define MFB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define MFB_API __declspec(dllexport)
#else
#define MFB_API __attribute__((visibility("default")))
#endif

/* Same handle type as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st* mfb_stream_t;

typedef enum mfb_status_t {
    MFB_OK = 0,
    MFB_EINVAL = 1,        /* bad argument: shape, stride, alias, pointer, option */
    MFB_ECUDA = 2,         /* a CUDA runtime/driver call failed (message: mfb_last_error) */
    MFB_ETIMEOUT = 3,      /* a bounded device-side wait gave up (see mfb_device_status) */
    MFB_ENCCL = 4,         /* an NCCL call failed */
    MFB_EUNSUPPORTED = 5,  /* valid request this build cannot serve (e.g. no sm_100 device) */
    MFB_ENOMEM = 6,        /* workspace allocation failed */
    MFB_ESHAPE = 7         /* operand shapes disagree (the reference's ShapeMismatchError) */
} mfb_status_t;

typedef enum mfb_precision_t {
    MFB_PRECISION_FP32 = 0, /* strict FP32 (default): error-compensated 3xTF32 on tcgen05 */
    MFB_PRECISION_TF32 = 1  /* single-pass TF32 inputs, FP32 accumulation */
} mfb_precision_t;

typedef enum mfb_epilogue_t {
    MFB_EPILOGUE_NONE = 0,
    MFB_EPILOGUE_BIAS = 1,      /* + bias[col] */
    MFB_EPILOGUE_BIAS_RELU = 2, /* relu(. + bias[col]) */
    MFB_EPILOGUE_BIAS_GELU = 3  /* tanh-GELU(. + bias[col]) */
} mfb_epilogue_t;

/*
 * C[m x n] = epilogue(alpha * op(A) * op(B) + beta * C).
 * op(A) is m x k: A is stored m x k (lda >= k) or, with trans_a, k x m (lda >= m).
 * op(B) is k x n: B is stored k x n (ldb >= n) or, with trans_b, n x k (ldb >= k).
 * ldc >= n. beta == 0 never reads C. k == 0 or alpha == 0 gives C = beta * C
 * followed by the epilogue (reference: implementation.inc:133-149).
 */
typedef struct mfb_gemm_desc {
    int m, n, k;
    int lda, ldb, ldc;
    float alpha, beta;
    int precision; /* mfb_precision_t */
    int trans_a, trans_b;
    int epilogue; /* mfb_epilogue_t */
} mfb_gemm_desc;

/* ---------------------------------------------------------------- status & errors */
MFB_API const char* mfb_status_string(mfb_status_t status);
/* Detail text of the last failure on the calling thread ("" when none). */
MFB_API const char* mfb_last_error(void);
/* Library version string and the kernel families compiled in. */
MFB_API const char* mfb_version(void);

/* Reads and clears the device status word that bounded waits report into.
 * *bits receives the raw word (0 = no timeout since the last read). Synchronizes
 * the device first. Returns MFB_ETIMEOUT when any bit was set. */
MFB_API mfb_status_t mfb_device_status(int device, uint32_t* bits);
/* Bound, in nanoseconds of device time, for every device-side wait of later launches
 * (default 4e9 = 4 s). Process-wide. */
MFB_API mfb_status_t mfb_set_wait_limit_ns(uint64_t limit_ns);
MFB_API uint64_t mfb_get_wait_limit_ns(void);
/* Synchronizes `stream` on `device`, then reports CUDA errors and device timeouts. */
MFB_API mfb_status_t mfb_sync(int device, mfb_stream_t stream);

/* ---------------------------------------------------------------- hw::cuda_gemm drop-in */
/* Asynchronous strict-FP32 GEMM on the device's internal stream (created lazily),
 * thread-safe through a per-device lock; wait with mfb_cuda_sync. Same arguments
 * and meaning as matrix_pro::hw::cuda_gemm (cuda_hooks.hpp:17-18). */
MFB_API mfb_status_t mfb_cuda_gemm(int device, int m, int n, int k, const float* a, int lda, const float* b,
                                   int ldb, float* c, int ldc, float alpha, float beta);
MFB_API mfb_status_t mfb_cuda_sync(int device);
MFB_API mfb_status_t mfb_cuda_device_count(int* count);

/* ---------------------------------------------------------------- one-shot GEMM */
/* Stream-ordered GEMM. Scratch (3xTF32 split planes, repacked operands) comes from a
 * per-(device, stream) cache that grows on demand; for allocation-free launches
 * (CUDA graph capture) create a plan. bias: n floats, required iff epilogue != NONE. */
MFB_API mfb_status_t mfb_sgemm(int device, mfb_stream_t stream, const mfb_gemm_desc* desc, const float* a,
                               const float* b, float* c, const float* bias);

/* ---------------------------------------------------------------- GEMM on host operands */
/* mfb_sgemm where each of A, B, C and bias may be host memory (pinned for full PCIe speed;
 * pageable works, staged by the driver) or memory of `device`: the GPU share of the
 * reference's host-side GEMM, HeterogeneousScheduler::gemm (src/hw/scheduler.cpp:236-312),
 * which copies B, A and C in, runs hw::cuda_gemm and copies C out one step after another.
 * Here B and the bias are copied once, and the rows of C stream through a ring of device
 * panels: copy-in of panel i, the GEMM of panel i-1 and copy-out of panel i-2 run at once
 * (two library-owned copy streams, the GEMM on `stream`). Stream-ordered: host C holds the
 * result once `stream` is synchronized. Device buffers are cached per device and grow on
 * demand; calls on one device are serialized. */
MFB_API mfb_status_t mfb_sgemm_host(int device, mfb_stream_t stream, const mfb_gemm_desc* desc, const float* a,
                                    const float* b, float* c, const float* bias);

/* ---------------------------------------------------------------- row-split GEMM over GPUs */
/* One block of rows of A and C on one GPU of this process. */
typedef struct mfb_row_block {
    int device;      /* CUDA device holding the block (one block per device) */
    int rows;        /* rows of A and C in the block (>= 0); the blocks' rows add up to desc->m */
    const float* a;  /* rows x k of A, row stride desc->lda, memory of `device` */
    float* c;        /* rows x n of C, row stride desc->ldc, memory of `device` */
} mfb_row_block;

/* C = epilogue(alpha * A * B + beta * C) over several GPUs: block r holds rows of A and C on
 * blocks[r].device (blocks in row order), B (k x n, row stride desc->ldb) and the bias (n
 * floats, iff epilogue != NONE) are memory of blocks[root].device. B and the bias reach the
 * other GPUs by NCCL broadcasts over NVLink/NVSwitch, B in column panels, and every GPU
 * multiplies the panels that have arrived while later ones are in flight; C stays split.
 * trans_a/trans_b must be 0; precision as mfb_sgemm. Blocking: work already queued on the
 * devices finishes first, and the call returns when every GPU is done. Calls are serialized.
 * The multi-GPU form of the GPU share of HeterogeneousScheduler::gemm (src/hw/scheduler.cpp:
 * 238-312: a block of rows on one device, B sent over PCIe) and of the host-staged broadcast
 * (src/hw/collectives.cpp:219-235). */
MFB_API mfb_status_t mfb_sgemm_multi(const mfb_row_block* blocks, int block_count, int root,
                                     const mfb_gemm_desc* desc, const float* b, const float* bias);

/* ---------------------------------------------------------------- strided-batched GEMM */
/* batch_count GEMMs that share one descriptor: C_i = epilogue(alpha op(A_i) op(B_i) + beta C_i)
 * with A_i = a + i*stride_a, B_i = b + i*stride_b, C_i = c + i*stride_c (strides in floats;
 * a stride of 0 reuses one operand for every entry). Replaces cublasSgemmStridedBatched in
 * batch_matmul (src/nn/batch.cu:12-35) and in its backward, batch_matmul_backward_left
 * (G x B^T: trans_b) and batch_matmul_backward_right (A^T x G: trans_a)
 * (src/nn/backward/batched_matmul.inc:7-55). All entries run in one tcgen05 launch; the
 * outputs may not overlap each other or any input. batch_count <= 65535. */
MFB_API mfb_status_t mfb_sgemm_strided_batched(int device, mfb_stream_t stream, const mfb_gemm_desc* desc,
                                               const float* a, long long stride_a, const float* b,
                                               long long stride_b, float* c, long long stride_c, int batch_count,
                                               const float* bias);

/* ---------------------------------------------------------------- allocation-free GEMM */
/* No counterpart in the reference. mfb_sgemm without any device allocation, for callers
 * that cannot allocate device memory when they call: code under a framework that owns
 * the device-memory budget, latency-critical paths where cudaMalloc/cudaFree (which
 * synchronize the device) or an out-of-memory failure mid-call are not acceptable, and
 * plugins that may not touch their host process's allocator. Same arguments and results
 * as mfb_sgemm (always the tcgen05 path, strict FP32 or TF32). The operand scratch is a
 * static device array of MFB_NOALLOC_SCRATCH_BYTES (64 MiB, e.g. a 2048^3 strict GEMM)
 * that every GPU loading the library holds until exit; larger problems return
 * MFB_EINVAL. The first call on a device looks up the array's address
 * (cudaGetSymbolAddress) and caches it for the device's current CUDA context; make that
 * call before any stream capture, and again after a device reset (a new context looks the
 * address up once more). All calls share the array and it keeps the last call's contents
 * (nothing in it needs to start at zero: the operand prepass rewrites all that the GEMM
 * reads): calls that overlap on the GPU race, so order them on one stream. Unlike
 * mfb_sgemm, vectors (n <= 16 or m == 1) also run the tcgen05 GEMM here. */
#define MFB_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
MFB_API mfb_status_t mfb_sgemm_noalloc(int device, mfb_stream_t stream, const mfb_gemm_desc* desc, const float* a,
                                       const float* b, float* c, const float* bias);

/* ---------------------------------------------------------------- plans */
typedef struct mfb_plan* mfb_plan_t;

typedef struct mfb_plan_info {
    int m, n, k;
    int precision, trans_a, trans_b, epilogue;
    int path;              /* 0 tcgen05 GEMM, 1 GEMV/skinny, 2 scale-only (k == 0), 3 empty (m or n == 0) */
    int tile_n;            /* tcgen05 tile width (128 x tile_n) */
    int stages;            /* shared-memory pipeline depth */
    int candidates;        /* tile configurations considered by mfb_plan_tune */
    size_t workspace_bytes;/* device scratch owned by the plan */
    char kernel[64];       /* kernel family name */
    int sm_pair;           /* 1: 256-row tiles on SM pairs (tcgen05.mma.cta_group::2) */
    int split_k;           /* most persistent workers that share one tile's K range (1: no split) */
    int stream_k_tiles;    /* tiles whose K range is shared (stream-K), summed by a fix-up kernel */
    int workers;           /* persistent CTAs (or SM pairs) of one launch */
} mfb_plan_info;

/* Builds tile choice, scratch and launch state for one problem on `device`.
 * Allocates all scratch now; execute allocates nothing and is graph-capturable.
 * desc->alpha/beta are ignored (they are execute arguments). */
MFB_API mfb_status_t mfb_plan_create(int device, const mfb_gemm_desc* desc, mfb_plan_t* out);
MFB_API mfb_status_t mfb_plan_execute(mfb_plan_t plan, mfb_stream_t stream, const float* a, const float* b,
                                      float* c, float alpha, float beta, const float* bias);
/* The two phases of mfb_plan_execute, for callers that reuse prepared operands or
 * time the phases: prepare runs the operand prepass (3xTF32 hi/lo split, or TF32
 * round-to-nearest) into the plan's scratch; multiply runs only the GEMM kernel on the
 * prepared operands (a/b are still passed; GEMV plans read them there). prepare with
 * a NULL operand skips that operand, so A can be prepared while B is still arriving. No
 * reference counterpart: GemmPlan::execute (gemm.hpp:47) is both phases in one call. */
MFB_API mfb_status_t mfb_plan_prepare(mfb_plan_t plan, mfb_stream_t stream, const float* a, const float* b);
MFB_API mfb_status_t mfb_plan_multiply(mfb_plan_t plan, mfb_stream_t stream, const float* a, const float* b,
                                       float* c, float alpha, float beta, const float* bias);
/* Column-range phases, for a caller that receives B in column blocks (the row-split GEMM
 * broadcasts B in contiguous column panels): prepare_cols splits B's columns [n0, n1),
 * given as their own k x (n1 - n0) matrix with row stride ldb, into the plan's B planes;
 * multiply_cols computes only C's columns [n0, n1) (A prepared by mfb_plan_prepare, the
 * columns' B by prepare_cols). tcgen05 plans with a non-transposed B; n0 and n1 (unless
 * n1 == n) multiples of 32. No reference counterpart. */
MFB_API mfb_status_t mfb_plan_prepare_cols(mfb_plan_t plan, mfb_stream_t stream, const float* b, int ldb,
                                           int n0, int n1);
MFB_API mfb_status_t mfb_plan_multiply_cols(mfb_plan_t plan, mfb_stream_t stream, const float* a, float* c,
                                            float alpha, float beta, const float* bias, int n0, int n1);
/* Caps the persistent GEMM grid at `sms` SMs (0 = all), leaving the rest to work that
 * must run concurrently, e.g. an NCCL broadcast of the next column panel of B. */
MFB_API mfb_status_t mfb_plan_set_sm_limit(mfb_plan_t plan, int sms);
/* Times every admissible tile configuration on `scratch_c` (an m x n buffer with ldc
 * of the plan; c is never touched), keeps the fastest, and reports it. Synchronizes. */
MFB_API mfb_status_t mfb_plan_tune(mfb_plan_t plan, mfb_stream_t stream, const float* a, const float* b,
                                   float* scratch_c, int repeats, int* candidates_tested, float* best_ms);
/* Makes candidate `index` (0 = the plan's own first choice, < info.candidates) the
 * configuration execute uses, as mfb_plan_tune does with the fastest one; for callers that
 * keep their own tuning results. No reference counterpart. */
MFB_API mfb_status_t mfb_plan_select_candidate(mfb_plan_t plan, int index);
MFB_API mfb_status_t mfb_plan_info_get(mfb_plan_t plan, mfb_plan_info* info);
MFB_API mfb_status_t mfb_plan_destroy(mfb_plan_t plan);

/* ---------------------------------------------------------------- conv2d backward */
/* Gradients of mfb_conv2d_fwd (same n, c, h, w, k, r, s, stride, pad; P, Q as there), NCHW:
 * dx (N,C,H,W) = dL/dx from dy (N,K,P,Q) and the filters (K,C,R,S); dw (K,C,R,S) = dL/dw from x and
 * dy; db (K) = dL/dbias, the sum of dy over images and positions. Stride 1: dx is the forward
 * implicit GEMM on the transposed, flipped filters (padding R-1-pad, S-1-pad), dw a tcgen05
 * implicit GEMM over (image, position) split across the SMs and reduced in a fixed order;
 * other strides and problems under 1e7 FLOP run direct FP32 kernels with the reference's loop
 * order. db is a fixed-order reduction. precision as mfb_precision_t. Outputs are overwritten;
 * n == 0 gives dw = 0, db = 0. */
MFB_API mfb_status_t mfb_conv2d_bwd_data(int device, mfb_stream_t stream, int n, int c, int h, int w, int k, int r,
                                         int s, int stride, int pad, const float* dy, const float* wgt, float* dx,
                                         int precision);
MFB_API mfb_status_t mfb_conv2d_bwd_filter(int device, mfb_stream_t stream, int n, int c, int h, int w, int k, int r,
                                           int s, int stride, int pad, const float* x, const float* dy, float* dw,
                                           int precision);
MFB_API mfb_status_t mfb_conv2d_bwd_bias(int device, mfb_stream_t stream, int n, int k, int p, int q, const float* dy,
                                         float* db);

/* ---------------------------------------------------------------- collectives */
/* One buffer per rank, all in this process (CollectiveBuffer of
 * include/matrix_pro/distributed/collectives.hpp:22-26; device = CUDA device index). */
typedef struct mfb_collective_buffer {
    float* data;
    size_t count;
    int device;
} mfb_collective_buffer;

typedef enum mfb_reduce_op { MFB_REDUCE_SUM = 0, MFB_REDUCE_MEAN = 1, MFB_REDUCE_MAX = 2 } mfb_reduce_op;

/* Blocking collectives with the reference's results in the reference's places (Mean = Sum x
 * the float 1/rank_count; reduce_scatter leaves rank r's chunk in front of the all-reduced
 * rest of its buffer; scatter/gather/all_gather move count_per_rank leading elements). Ranks
 * on distinct GPUs run on one cached NCCL communicator per device set over NVLink/NVSwitch;
 * ranks all on one GPU run device-local copies and a fixed-order reduction. Any other
 * placement is MFB_EUNSUPPORTED. algorithm (0 ring, 1 tree) is accepted for compatibility;
 * NCCL chooses its own. Work already queued on the devices finishes before the collective. */
MFB_API mfb_status_t mfb_all_reduce(const mfb_collective_buffer* ranks, int rank_count, int op, int algorithm);
MFB_API mfb_status_t mfb_broadcast(const mfb_collective_buffer* ranks, int rank_count, int root);
MFB_API mfb_status_t mfb_all_gather(const mfb_collective_buffer* ranks, int rank_count, size_t count_per_rank);
MFB_API mfb_status_t mfb_reduce_scatter(const mfb_collective_buffer* ranks, int rank_count, int op);
MFB_API mfb_status_t mfb_scatter(const mfb_collective_buffer* ranks, int rank_count, int root, size_t count_per_rank);
MFB_API mfb_status_t mfb_gather(const mfb_collective_buffer* ranks, int rank_count, int root, size_t count_per_rank);
/* hw::cuda_nccl_allreduce: in-place all-reduce of ptrs[r] (count floats on devices[r]); op as above. */
MFB_API mfb_status_t mfb_cuda_nccl_allreduce(float** ptrs, const int* devices, int rank_count, size_t count,
                                             int reduce_op);

/* ---------------------------------------------------------------- covariance / correlation */
/* cov (cols x cols, row stride ldcov) = X_c^T X_c / max(rows - 1, 1), X_c = X minus its column
 * means, X rows x cols with row stride ldx; correlation divides by sqrt(cov_ii cov_jj) (1 on the
 * diagonal, 0 where a variance is not positive). Replaces matrix_pro::covariance / correlation
 * (src/ops/reductions/covariance.inc:23-60; the product ran on cublasSgemm, :38-44). The means
 * are one GEMV, the centering happens inside the GEMM's operand prepass, the product is the
 * tcgen05 GEMM (precision: MFB_PRECISION_FP32 strict or MFB_PRECISION_TF32). rows or cols == 0:
 * nothing is written. Scratch comes from the per-(device, stream) cache. */
MFB_API mfb_status_t mfb_covariance(int device, mfb_stream_t stream, int rows, int cols, const float* x, int ldx,
                                    float* cov, int ldcov, int precision);
MFB_API mfb_status_t mfb_correlation(int device, mfb_stream_t stream, int rows, int cols, const float* x, int ldx,
                                     float* corr, int ldcorr, int precision);

/* ---------------------------------------------------------------- GEMV / skinny */
/* Bandwidth-bound FP32 kernel for n <= 16 (y = A x with ldb/ldc strides) and for
 * m == 1 (row vector times matrix). Strict FP32 FMA arithmetic; trans_a/trans_b must
 * be 0. alpha/beta/epilogue as mfb_sgemm. */
MFB_API mfb_status_t mfb_gemv(int device, mfb_stream_t stream, const mfb_gemm_desc* desc, const float* a,
                              const float* b, float* c, const float* bias);

/* ---------------------------------------------------------------- conv2d forward */
/* NCHW cross-correlation: x (N,C,H,W), w (K,C,R,S), bias (K), y (N,K,P,Q) with
 * P = (H + 2 pad - R) / stride + 1, Q = (W + 2 pad - S) / stride + 1.
 * precision as mfb_precision_t. Scratch from the per-(device, stream) cache. */
MFB_API mfb_status_t mfb_conv2d_fwd(int device, mfb_stream_t stream, int n, int c, int h, int w, int k, int r,
                                    int s, int stride, int pad, const float* x, const float* wgt,
                                    const float* bias, float* y, int precision);

/* ---------------------------------------------------------------- device oracle */
/* One thread per output, FP32 FMA chain over k in order: a slow correctness oracle
 * that runs on the device (same desc semantics, no transposes). */
MFB_API mfb_status_t mfb_naive_sgemm(int device, mfb_stream_t stream, const mfb_gemm_desc* desc, const float* a,
                                     const float* b, float* c, const float* bias);

/* ---------------------------------------------------------------- failure-path probe */
/* Diagnostic (no reference counterpart): the TF32 tcgen05 MMA rate of `device` in TFLOP/s,
 * measured with back-to-back M = 128, N = n (64, 128 or 256), K = 8 MMAs on every SM from
 * reused shared-memory operands: the tensor pipe's ceiling for roofline denominators (a
 * streaming kernel also pays for operand fetch). Synchronous; takes a few milliseconds. */
MFB_API mfb_status_t mfb_probe_tf32_mma_tflops(int device, int n, float* tflops);

/* Launches a kernel that waits on an mbarrier nothing arrives on, bounded by
 * limit_ns; it records kStatusTimeoutProbe in the status word and returns. Used by
 * tests to exercise the timeout path without faulting or hanging the GPU. */
MFB_API mfb_status_t mfb_probe_wait_timeout(int device, mfb_stream_t stream, uint64_t limit_ns);

#ifdef __cplusplus
}
#endif

#endif /* MFB_H_ */
