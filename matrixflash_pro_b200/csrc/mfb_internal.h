// Host-side internals shared by the translation units of libmfb.so.
#pragma once

#include "../../include/mfb.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace mfb {

// Records `msg` as the calling thread's mfb_last_error() text and returns `status`.
mfb_status_t fail(mfb_status_t status, const std::string& msg);
mfb_status_t cuda_fail(cudaError_t err, const char* what);
void clear_error();

#define MFB_CUDA_TRY(expr, what)                                    \
    do {                                                            \
        cudaError_t mfb_err_ = (expr);                              \
        if (mfb_err_ != cudaSuccess) return ::mfb::cuda_fail(mfb_err_, what); \
    } while (0)

#define MFB_TRY(expr)                          \
    do {                                       \
        mfb_status_t mfb_st_ = (expr);         \
        if (mfb_st_ != MFB_OK) return mfb_st_; \
    } while (0)

// Restores the caller's current device on scope exit.
class DeviceGuard {
public:
    DeviceGuard() { cudaGetDevice(&saved_); }
    ~DeviceGuard() { cudaSetDevice(saved_); }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;

private:
    int saved_ = 0;
};

// Makes `device` current after checking it exists and is an sm_100 part.
mfb_status_t select_device(int device);
int sm_count(int device);
// SM count of the current device: the grid caps of the grid-stride kernels are multiples of it.
inline int current_sm_count() {
    int device = 0;
    cudaGetDevice(&device);
    return sm_count(device);
}
uint64_t wait_limit_ns();
bool stream_capturing(cudaStream_t stream);

// Scratch memory: per-(device, stream) grow-only buffers for calls without a plan.
mfb_status_t stream_workspace(int device, cudaStream_t stream, size_t bytes, void** out);

// Validates a GEMM description (shapes, strides, options) against the reference's rules.
mfb_status_t validate_desc(const mfb_gemm_desc* d, const float* a, const float* b, const float* c,
                           const float* bias, bool need_bias_check);

// ---------------------------------------------------------------------- tcgen05 GEMM
struct TcConfig {
    int bn = 128;
    int stages = 3;
    int planes = 2;   // 2 = strict 3xTF32, 1 = TF32
    int a_mn = 0;     // A stored transposed (MN-major)
    int b_mn = 1;     // B stored untransposed (MN-major)
    int pair = 0;     // 1: SM-pair kernel (cta_group::2, 256 x bn tiles)
    int stream_k = 0; // 1: the last tiles may share their K blocks among all workers (stream-K)
};

// How one launch of a configuration spreads its tiles over the persistent workers.
struct TcSchedule {
    long long tiles = 0;
    int kb = 0;              // K blocks per tile
    int workers = 0;         // CTAs (single-CTA tiles) or SM pairs
    int sk_tiles = 0;        // tiles whose K blocks are shared (stream-K); 0 = all data parallel
    int split = 1;           // most workers sharing one tile
    size_t partial_bytes = 0;  // partial slots a stream-K launch needs (2 per worker)
};

// Admissible tile configurations for a problem, best-guess first.
// Strided batch of GEMMs sharing one descriptor: entry i reads A + i*stride_a and
// B + i*stride_b and writes C + i*stride_c (strides in floats).
struct TcBatch {
    int count = 1;
    long long stride_a = 0, stride_b = 0, stride_c = 0;
};

// Optional transform applied by the operand prepass: subtract shift[column of the stored
// matrix] from every element of A and/or B before the TF32 split (covariance centering).
struct TcPrologue {
    const float* a_col_shift = nullptr;
    const float* b_col_shift = nullptr;
    // A and B are the same stored matrix with the same shift (X^T X): one prepass, and both
    // operand maps read the same planes.
    bool shared_planes = false;
};

// Column range [n0, n1) of a non-transposed B (n1 < 0: up to n). The prepare phase then
// splits B's columns [n0, n1) from `b_src` (k x (n1 - n0), row stride b_ld) into the
// planes' columns [n0, n1); the multiply phase computes only C's columns [n0, n1).
// n0 is a multiple of 32.
struct TcColumns {
    int n0 = 0;
    int n1 = -1;
    const float* b_src = nullptr;
    long long b_ld = 0;
};

// Tile configurations for `d`, best first (SM-pair 256 x 256 tiles when they fill the GPU,
// for single GEMMs and strided batches alike).
int tc_candidates(const mfb_gemm_desc& d, TcConfig* out, int max_out, int batch = 1);

// Scratch the tcgen05 path needs for `d`: hi/lo planes of A and B (strict) or one
// rounded TF32 plane of each (TF32), rows padded to 16 bytes.
size_t tc_workspace_bytes(const mfb_gemm_desc& d, int batch = 1);
// The planes (256-byte aligned) plus the partial slots of a stream-K launch of `cfg` on all
// workers of the current device. A launch given less runs every tile data parallel.
size_t tc_workspace_bytes_for(const mfb_gemm_desc& d, const TcConfig& cfg, int batch = 1);
// The schedule a launch of `cfg` over n_cols output columns gets on `dev` (sm_limit as tc_gemm).
mfb_status_t tc_schedule(const mfb_gemm_desc& d, const TcConfig& cfg, int dev, int sm_limit, int batch, int n_cols,
                         TcSchedule* out);

// Runs the tcgen05 GEMM on `stream`: kPhasePrepare launches the split/round prepass of
// the operands into `workspace`, kPhaseMultiply the GEMM kernel on the prepared
// operands. sm_limit > 0 caps the persistent grid.
enum { kPhasePrepare = 1, kPhaseMultiply = 2, kPhaseAll = 3 };
mfb_status_t tc_gemm(const mfb_gemm_desc& d, const TcConfig& cfg, cudaStream_t stream, const float* a,
                     const float* b, float* c, const float* bias, void* workspace, size_t workspace_bytes,
                     int phases = kPhaseAll, int sm_limit = 0, const TcBatch& batch = TcBatch(),
                     const TcPrologue& prologue = TcPrologue(), const TcColumns& cols = TcColumns());

// cuTensorMapEncodeTiled for FP32 tensors of rank <= 5 (no interleave, L2 256B promotion,
// zero fill out of bounds); strides_bytes has rank - 1 entries.
mfb_status_t encode_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle);

// C = beta * C, then the epilogue; the k == 0 / alpha == 0 path.
mfb_status_t scale_output(const mfb_gemm_desc& d, cudaStream_t stream, float* c, const float* bias);

// ---------------------------------------------------------------------- GEMV
bool gemv_eligible(const mfb_gemm_desc& d);
size_t gemv_workspace_bytes(const mfb_gemm_desc& d);
mfb_status_t gemv_launch(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                         const float* bias, void* workspace, size_t workspace_bytes);

// ---------------------------------------------------------------------- conv
// conv2d backward (conv.cu): input gradient, weight gradient, bias gradient.
mfb_status_t conv2d_bwd_data_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r, int s,
                                    int stride, int pad, const float* dy, const float* wgt, float* dx, int precision);
mfb_status_t conv2d_bwd_filter_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r,
                                      int s, int stride, int pad, const float* x, const float* dy, float* dw,
                                      int precision);
mfb_status_t conv2d_bwd_bias_launch(int device, cudaStream_t stream, int n, int k, int P, int Q, const float* dy,
                                    float* db);
mfb_status_t conv2d_launch(int device, cudaStream_t stream, int n, int c, int h, int w, int k, int r, int s,
                           int stride, int pad, const float* x, const float* wgt, const float* bias, float* y,
                           int precision);

// ---------------------------------------------------------------------- NCCL (collectives.cu)
// The cached communicator set (ncclCommInitAll) of a list of distinct devices of this process:
// its per-device non-blocking streams, in device-list order.
mfb_status_t nccl_streams(const std::vector<int>& devices, std::vector<cudaStream_t>* streams);
// In-place ncclBroadcast of `count` floats from bufs[root] into every bufs[r] (on devices[r]), one
// NCCL group, enqueued on the set's streams; returns without waiting.
mfb_status_t nccl_broadcast_group(const std::vector<int>& devices, const std::vector<float*>& bufs, size_t count,
                                  int root);

// ---------------------------------------------------------------------- naive
mfb_status_t naive_launch(const mfb_gemm_desc& d, cudaStream_t stream, const float* a, const float* b, float* c,
                          const float* bias);

// ---------------------------------------------------------------------- probes
mfb_status_t probe_wait_launch(cudaStream_t stream, uint64_t limit_ns);
mfb_status_t read_and_clear_status(uint32_t* bits);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace mfb
