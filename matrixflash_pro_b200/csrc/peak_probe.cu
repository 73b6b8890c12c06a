// Diagnostic: the TF32 tcgen05 MMA rate of this GPU, measured, for roofline denominators.
//
// One CTA per SM; one thread issues back-to-back tcgen05.mma.cta_group::1.kind::tf32
// (M = 128, N as asked, K = 8) from one zero-filled shared-memory A/B pair into TMEM,
// committing every kProbeMmasPerCommit MMAs. Operands are reused, so this is the tensor
// pipe's issue/compute ceiling, not what a streaming kernel can reach (its MMAs also fetch
// operands from shared memory). Bounded waits as everywhere else.
#include "mfb_internal.h"
#include "tc_kernel.cuh"

namespace mfb {
namespace {

constexpr int kProbeMmasPerCommit = 48;

template <int N>
__global__ void __launch_bounds__(128, 1) tf32_mma_rate_kernel(int iterations, unsigned long long limit_ns) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a = smem;          // 128 rows x 128 B
    uint8_t* b = smem + 16384;  // N rows x 128 B
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + N * 128);
    uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
    const int warp = threadIdx.x / 32;
    for (int i = threadIdx.x; i < (16384 + N * 128) / 4; i += blockDim.x) reinterpret_cast<float*>(smem)[i] = 0.0f;
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    if (warp == 0) {
        tmem_alloc(slot, N < 32 ? 32 : N);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *slot;
    if (threadIdx.x == 0) {
        constexpr uint32_t idesc = umma_idesc_tf32(128, N, 0, 0);
        uint32_t phase = 0;
        for (int it = 0; it < iterations; ++it) {
            for (int j = 0; j < kProbeMmasPerCommit; ++j) {
                const int ks = j & 3;
                umma_tf32(tmem, umma_smem_desc(smem_u32(a) + ks * 32, 16, 1024, kLayoutSwizzle128B),
                          umma_smem_desc(smem_u32(b) + ks * 32, 16, 1024, kLayoutSwizzle128B), idesc, 1u);
            }
            umma_commit(bar);
            if (!mbar_wait_bounded(bar, phase, limit_ns, nullptr)) {
                report_status(kStatusTimeoutProbe, nullptr);
                // let the MMAs still in flight retire before TMEM is freed
                umma_commit(bar);
                mbar_wait_drain(bar, phase ^ 1, limit_ns);
                break;
            }
            phase ^= 1;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, N < 32 ? 32 : N);
    }
}

template <int N>
mfb_status_t run_rate_probe(int device, float* tflops) {
    constexpr int smem = 1024 + 16384 + N * 128 + 64;
    auto fn = tf32_mma_rate_kernel<N>;
    MFB_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem), "probe smem attribute");
    const int sms = sm_count(device);
    cudaStream_t stream = nullptr;
    MFB_CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "probe stream");
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    const int iterations = 2000;
    fn<<<sms, 128, smem, stream>>>(20, wait_limit_ns());  // warm-up: clocks up, code loaded
    cudaEventRecord(e0, stream);
    fn<<<sms, 128, smem, stream>>>(iterations, wait_limit_ns());
    cudaEventRecord(e1, stream);
    cudaError_t err = cudaEventSynchronize(e1);
    float ms = 0.0f;
    if (err == cudaSuccess) err = cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(stream);
    MFB_CUDA_TRY(err, "probe timing");
    MFB_CUDA_TRY(cudaGetLastError(), "probe launch");
    const double flops = 2.0 * 128 * N * 8 * static_cast<double>(kProbeMmasPerCommit) * iterations * sms;
    *tflops = ms > 0.0f ? static_cast<float>(flops / (ms * 1e-3) / 1e12) : 0.0f;
    return read_and_clear_status(nullptr);
}

}  // namespace
}  // namespace mfb

extern "C" MFB_API mfb_status_t mfb_probe_tf32_mma_tflops(int device, int n, float* tflops) {
    mfb::clear_error();
    if (!tflops) return mfb::fail(MFB_EINVAL, "null output pointer");
    mfb::DeviceGuard guard;
    MFB_TRY(mfb::select_device(device));
    switch (n) {
        case 64: return mfb::run_rate_probe<64>(device, tflops);
        case 128: return mfb::run_rate_probe<128>(device, tflops);
        case 256: return mfb::run_rate_probe<256>(device, tflops);
        default: return mfb::fail(MFB_EINVAL, "probe N must be 64, 128 or 256");
    }
}
