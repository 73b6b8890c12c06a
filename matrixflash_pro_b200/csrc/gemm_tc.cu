// Host side of the tcgen05 GEMM: operand preparation (3xTF32 hi/lo split planes, or
// one round-to-nearest TF32 plane per operand), TMA descriptor encoding,
// tile-configuration choice and launch. The reference's cuBLAS/cuBLASLt bodies
// this replaces: src/hw/cuda_backend.cu:91-99 and
// src/ops/gemm/plan/implementation.inc:111-151.
#include "gemm_tc.cuh"
#include "mfb_internal.h"
#include "tc_pair_kernel.cuh"

#include <algorithm>
#include <cstring>
#include <map>
#include <mutex>

namespace mfb {

// ------------------------------------------------------------------------------------
// Prepass kernels (HBM-bound, 128-bit accesses where the layout allows)
// ------------------------------------------------------------------------------------

__device__ __forceinline__ float round_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// hi = tf32(x) (round to nearest), lo = tf32(x - hi); x - hi is exact in FP32, so
// hi + lo carries 22 significant bits of x. lo == nullptr writes only hi: the TF32
// mode's operands, rounded to nearest like cuBLAS/CUTLASS TF32 conversion (the tensor
// core itself would truncate the low 13 bits, a bias that shows on same-sign data).
// One operand's prepass: rows x cols of x (row stride ldx) into plane(s) of row stride ldp;
// blockIdx.y walks a strided batch (source y at x + y * x_batch, planes at hi/lo + y * p_batch);
// shift (nullable, one value per stored column) is subtracted first (covariance centering).
struct SplitJob {
    const float* x;
    long long ldx;
    int rows, cols;
    float* hi;
    float* lo;
    long long ldp;
    int vec_in;
    long long x_batch, p_batch;
    const float* shift;
    int blocks;  // blocks of the launch's x dimension that serve this job
    long long wcols;  // columns written per plane row (multiple of 4, <= ldp); zeros past `cols`
};

__device__ __forceinline__ void split_tf32_job(const SplitJob& j, int block, int nblocks) {
    const float* x = j.x + blockIdx.y * j.x_batch;
    float* hi = j.hi + blockIdx.y * j.p_batch;
    float* lo = j.lo != nullptr ? j.lo + blockIdx.y * j.p_batch : nullptr;
    const long long groups_per_row = j.wcols / 4;
    const long long total = static_cast<long long>(j.rows) * groups_per_row;
    for (long long idx = block * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(nblocks) * blockDim.x) {
        const long long r = idx / groups_per_row;
        const int c0 = static_cast<int>(idx - r * groups_per_row) * 4;
        const float* src = x + r * j.ldx + c0;
        float v[4];
        if (j.vec_in && c0 + 3 < j.cols) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(src));
            v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
        } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = (c0 + e < j.cols) ? __ldg(src + e) : 0.0f;
        }
        if (j.shift != nullptr) {
#pragma unroll
            for (int e = 0; e < 4; ++e) v[e] = (c0 + e < j.cols) ? v[e] - __ldg(j.shift + c0 + e) : 0.0f;
        }
        float4 h, l;
        if (lo != nullptr) {
            float hv[4], lv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                hv[e] = round_tf32(v[e]);
                lv[e] = round_tf32(v[e] - hv[e]);
            }
            h = make_float4(hv[0], hv[1], hv[2], hv[3]);
            l = make_float4(lv[0], lv[1], lv[2], lv[3]);
            *reinterpret_cast<float4*>(lo + r * j.ldp + c0) = l;
        } else {
            h = make_float4(round_tf32(v[0]), round_tf32(v[1]), round_tf32(v[2]), round_tf32(v[3]));
        }
        *reinterpret_cast<float4*>(hi + r * j.ldp + c0) = h;
    }
}

// Both operands' prepasses in one launch: blocks [0, a.blocks) serve A, the rest B.
__global__ void split_tf32_kernel(SplitJob a, SplitJob b) {
    grid_launch_dependents();  // the GEMM that follows may set up while this grid drains
    if (static_cast<int>(blockIdx.x) < a.blocks)
        split_tf32_job(a, blockIdx.x, a.blocks);
    else
        split_tf32_job(b, blockIdx.x - a.blocks, b.blocks);
}

// C = beta * C (beta == 0 writes zeros without reading), then the column-bias epilogue.
// Mirrors scale_output + apply_epilogue of the reference (plan/epilogue.cuh:20,
// gemm_fused.cu:23-60) for the k == 0 / alpha == 0 case.
__global__ void scale_epilogue_kernel(float* __restrict__ c, long long ldc, int m, int n, float beta,
                                      const float* __restrict__ bias, int epilogue) {
    const long long total = static_cast<long long>(m) * n;
    for (long long idx = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; idx < total;
         idx += static_cast<long long>(gridDim.x) * blockDim.x) {
        const long long r = idx / n;
        const int col = static_cast<int>(idx - r * n);
        float* p = c + r * ldc + col;
        const float v = beta == 0.0f ? 0.0f : beta * *p;
        *p = apply_epilogue_op(v, bias, col, epilogue);
    }
}

// Stream-K fix-up: every tile whose K blocks were shared by several workers (see
// TcWorkIter) is the sum of its partial slots, added in K order (worker order), then
// written through the GEMM's own store (alpha, beta * C, bias, activation). Tiles that one
// worker covered whole were written by the GEMM and are skipped. blockIdx.y = stream-K
// tile; the x blocks split its ROWS x BN values, four consecutive columns per thread.
// Workers w0 < w <= w1 of a shared tile r start their ranges inside it, so they hold it in
// slot 2w; only w0 may have started in an earlier tile (slot 2 w0 + 1). Thread 0 finds
// w0, w1 and that first slot once per block.
template <class Prob, int ROWS>
__global__ void __launch_bounds__(256) streamk_reduce_kernel(const GemmTcParams p, int workers) {
    constexpr int BN = Prob::BN;
    constexpr int kGroupsPerRow = BN / 4;
    __shared__ int s_w0, s_w1, s_first_slot;
    grid_dependency_wait();  // the GEMM's partial sums (programmatic launch)
    const int r = blockIdx.y;
    if (threadIdx.x == 0) {
        const int kb = p.num_kb;
        const long long iters = static_cast<long long>(p.sk_tiles) * kb;
        const int w0 = tc_sk_owner(static_cast<long long>(r) * kb, iters, workers);
        s_w0 = w0;
        s_w1 = tc_sk_owner(static_cast<long long>(r + 1) * kb - 1, iters, workers);
        s_first_slot = (iters * w0 / workers) / kb == r ? 2 * w0 : 2 * w0 + 1;
    }
    __syncthreads();
    const int w0 = s_w0, w1 = s_w1;
    if (w0 == w1) return;
    const int first_slot = s_first_slot;
    const typename Prob::Tile t = Prob::tile(p, Prob::num_tiles(p) - p.sk_tiles + r);
    using Store = GemmProblem<BN, 1, 1, 0, 1>;
    const typename Store::Tile st{t.m0, t.n0, t.b};
    const int rows = min(ROWS, p.m - t.m0);
    const int cols = min(BN, p.n - t.n0);
    constexpr size_t kSlot = static_cast<size_t>(ROWS) * BN;
    for (int g = blockIdx.x * blockDim.x + threadIdx.x; g < ROWS * kGroupsPerRow; g += gridDim.x * blockDim.x) {
        const int row = g / kGroupsPerRow;
        const int col = (g % kGroupsPerRow) * 4;
        if (row >= rows || col >= cols) continue;
        const size_t off = static_cast<size_t>(row) * BN + col;
        auto slot_at = [&](int w) {
            return *reinterpret_cast<const float4*>(p.partials + static_cast<size_t>(2 * w) * kSlot + off);
        };
        auto add = [](float4& a, const float4& v) {
            a.x += v.x;
            a.y += v.y;
            a.z += v.z;
            a.w += v.w;
        };
        float4 acc = *reinterpret_cast<const float4*>(p.partials + first_slot * kSlot + off);
        int w = w0 + 1;
        // Four shares' loads in flight at a time; the adds stay in K order.
        for (; w + 3 <= w1; w += 4) {
            const float4 v0 = slot_at(w), v1 = slot_at(w + 1), v2 = slot_at(w + 2), v3 = slot_at(w + 3);
            add(acc, v0);
            add(acc, v1);
            add(acc, v2);
            add(acc, v3);
        }
        for (; w <= w1; ++w) add(acc, slot_at(w));
        const float out[4] = {acc.x, acc.y, acc.z, acc.w};
        Store::template store<4>(p, st, row, col, out);
    }
}

// ------------------------------------------------------------------------------------
// TMA descriptors
// ------------------------------------------------------------------------------------
namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Map over a stored row-major matrix (cols contiguous) with outer batch and plane axes:
// 4-D (cols, rows, batch, plane), for the single-CTA and the SM-pair kernels alike. K-major
// tiles use the 128B swizzle with 16-byte atoms; MN-major TF32 tiles the 128B swizzle with
// 32-byte atoms, the only shared-memory layout tcgen05 accepts for them.
mfb_status_t encode_operand(CUtensorMap* map, const float* base, int rows, int cols, long long ld, int planes,
                            long long plane_stride_floats, int box_cols, int box_rows, bool mn_major,
                            int batch = 1, long long batch_stride_floats = 0) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(MFB_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
    const long long plane_stride = plane_stride_floats > 0 ? plane_stride_floats : ld * static_cast<long long>(rows);
    const long long batch_stride = batch_stride_floats > 0 ? batch_stride_floats : ld * static_cast<long long>(rows);
    const int rank = 4;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows),
                          static_cast<cuuint64_t>(batch), static_cast<cuuint64_t>(planes)};
    cuuint64_t strides[3] = {static_cast<cuuint64_t>(ld) * 4, static_cast<cuuint64_t>(batch_stride) * 4,
                             static_cast<cuuint64_t>(plane_stride) * 4};
    cuuint32_t box[4] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1,
                         static_cast<cuuint32_t>(planes)};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, static_cast<cuuint32_t>(rank), const_cast<float*>(base),
                    dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE,
                    mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(MFB_ECUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")");
    return MFB_OK;
}

}  // namespace

mfb_status_t encode_tensor_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                               const uint64_t* strides_bytes, const uint32_t* box, CUtensorMapSwizzle swizzle) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return fail(MFB_ECUDA, "cuTensorMapEncodeTiled entry point unavailable");
    cuuint64_t d[5];
    cuuint64_t st[4];
    cuuint32_t b[5];
    cuuint32_t es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        es[i] = 1;
        if (i + 1 < rank) st[i] = strides_bytes[i];
    }
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st,
                    b, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(MFB_ECUDA, "cuTensorMapEncodeTiled failed (code " + std::to_string(static_cast<int>(r)) + ")");
    return MFB_OK;
}

namespace {

// ------------------------------------------------------------------------------------
// Kernel table
// ------------------------------------------------------------------------------------

struct TcEntry {
    int bn, stages, planes, a_mn, b_mn;
    const void* fn;
    int smem;
    int threads;
    int pair;  // SM-pair kernel (cluster of 2, 256-row tiles)
    int kslabs;  // 32-deep K slabs per stage (the kernel's K block is 32 * kslabs deep)
    const void* reduce;  // stream-K fix-up kernel for this tile shape
};

template <int BN, int STAGES, int PLANES, int A_MN, int B_MN, int KS = 1>
TcEntry make_entry() {
    using P = GemmProblem<BN, STAGES, PLANES, A_MN, B_MN, KS>;
    using L = TcLayout<P>;
    return TcEntry{BN, STAGES, PLANES, A_MN, B_MN, reinterpret_cast<const void*>(&tc_persistent_kernel<P>), L::kBytes,
                   L::kThreads, 0, KS, reinterpret_cast<const void*>(&streamk_reduce_kernel<P, kTcBM>)};
}

template <int BN, int STAGES, int PLANES, int A_MN, int B_MN, int KS = 1>
TcEntry make_pair_entry() {
    using P = GemmPairProblem<BN, STAGES, PLANES, A_MN, B_MN, KS>;
    using L = TcPairLayout<P>;
    return TcEntry{BN, STAGES, PLANES, A_MN, B_MN, reinterpret_cast<const void*>(&tc_pair_kernel<P>), L::kBytes,
                   L::kThreads, 1, KS, reinterpret_cast<const void*>(&streamk_reduce_kernel<P, 2 * kTcBM>)};
}

const TcEntry* kernel_table(int* count) {
    static const TcEntry table[] = {
        // SM pairs, 256 x 256 tiles: strict and TF32, every transpose combination
        make_pair_entry<256, 3, 2, 0, 1>(),
        make_pair_entry<256, 3, 1, 0, 1, 2>(),
        make_pair_entry<256, 3, 2, 1, 1>(),
        make_pair_entry<256, 3, 1, 1, 1, 2>(),
        make_pair_entry<256, 3, 2, 0, 0>(),
        make_pair_entry<256, 3, 1, 0, 0, 2>(),
        make_pair_entry<256, 3, 2, 1, 0>(),
        make_pair_entry<256, 3, 1, 1, 0, 2>(),
        // strict FP32 (3xTF32 split planes, chunked round-to-nearest accumulation)
        make_entry<256, 2, 2, 0, 1>(),
        make_entry<128, 3, 2, 0, 1>(),
        make_entry<64, 2, 2, 0, 1, 2>(),
        make_entry<128, 3, 2, 1, 1>(),
        make_entry<128, 3, 2, 0, 0>(),
        make_entry<128, 3, 2, 1, 0>(),
        // TF32 single pass
        make_entry<256, 2, 1, 0, 1, 2>(),
        make_entry<128, 3, 1, 0, 1, 2>(),
        make_entry<64, 4, 1, 0, 1, 2>(),
        make_entry<128, 3, 1, 1, 1, 2>(),
        make_entry<128, 3, 1, 0, 0, 2>(),
        make_entry<128, 3, 1, 1, 0, 2>(),
    };
    *count = static_cast<int>(sizeof(table) / sizeof(table[0]));
    return table;
}

const TcEntry* find_kernel(const TcConfig& c) {
    int count = 0;
    const TcEntry* t = kernel_table(&count);
    for (int i = 0; i < count; ++i)
        if (t[i].bn == c.bn && t[i].stages == c.stages && t[i].planes == c.planes && t[i].a_mn == c.a_mn &&
            t[i].b_mn == c.b_mn && t[i].pair == c.pair)
            return &t[i];
    return nullptr;
}

long long round_up(long long v, long long q) { return (v + q - 1) / q * q; }

struct PreparedOperand {
    const float* base = nullptr;
    int rows = 0, cols = 0;
    long long ld = 0;
    long long plane_stride = 0;  // floats; 0 when one plane
    long long batch_stride = 0;  // floats between batch entries of one plane
    bool needs_prepass = false;
};

// Stored-matrix geometry of op(A) / op(B).
void stored_dims(const mfb_gemm_desc& d, bool is_a, int* rows, int* cols, long long* ld) {
    if (is_a) {
        *rows = d.trans_a ? d.k : d.m;
        *cols = d.trans_a ? d.m : d.k;
        *ld = d.lda;
    } else {
        *rows = d.trans_b ? d.n : d.k;
        *cols = d.trans_b ? d.k : d.n;
        *ld = d.ldb;
    }
}

size_t plane_floats(int rows, int cols) {
    return static_cast<size_t>(round_up(static_cast<long long>(rows) * round_up(cols, 4), 64));
}

}  // namespace

// ------------------------------------------------------------------------------------
// Configuration choice
// ------------------------------------------------------------------------------------
namespace {

// Serialized: the attributes are per kernel, and concurrent host threads launch the same ones.
std::mutex g_attr_mutex;

mfb_status_t set_kernel_attributes(const TcEntry* e) {
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    MFB_CUDA_TRY(cudaFuncSetAttribute(e->fn, cudaFuncAttributeMaxDynamicSharedMemorySize, e->smem),
                 "cudaFuncSetAttribute(max dynamic smem)");
    if (e->pair)
        MFB_CUDA_TRY(cudaFuncSetAttribute(e->fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 0),
                     "cudaFuncSetAttribute(cluster size)");
    return MFB_OK;
}

// Clusters of 2 CTAs of the pair kernel `e` that can be co-resident on `dev` (queried once).
mfb_status_t pair_capacity(const TcEntry* e, int dev, int* out) {
    static std::mutex mutex;
    static std::map<std::pair<int, const void*>, int> cache;
    {
        std::lock_guard<std::mutex> lock(mutex);
        auto it = cache.find({dev, e->fn});
        if (it != cache.end()) {
            *out = it->second;
            return MFB_OK;
        }
    }
    MFB_TRY(set_kernel_attributes(e));
    cudaLaunchConfig_t lc{};
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    lc.gridDim = dim3(static_cast<unsigned>(2 * (sm_count(dev) / 2)));
    lc.blockDim = dim3(e->threads);
    lc.dynamicSmemBytes = static_cast<size_t>(e->smem);
    lc.attrs = &attr;
    lc.numAttrs = 1;
    int n = 0;
    MFB_CUDA_TRY(cudaOccupancyMaxActiveClusters(&n, e->fn, &lc), "cudaOccupancyMaxActiveClusters");
    if (n <= 0) return fail(MFB_EUNSUPPORTED, "no SM pair can host the pair GEMM kernel");
    std::lock_guard<std::mutex> lock(mutex);
    cache[{dev, e->fn}] = n;
    *out = n;
    return MFB_OK;
}

// Persistent workers of a launch of `e`: one per SM (single-CTA tiles) or per co-resident SM
// pair, within the caller's SM limit.
mfb_status_t worker_count(const TcEntry* e, int dev, int sm_limit, int* out) {
    const int sms = sm_limit > 0 ? std::min(sm_limit, sm_count(dev)) : sm_count(dev);
    if (!e->pair) {
        *out = std::max(1, sms);
        return MFB_OK;
    }
    int cap = 0;
    MFB_TRY(pair_capacity(e, dev, &cap));
    *out = std::max(1, std::min(cap, sms / 2));
    return MFB_OK;
}

// Stream-K share of a launch: how many of the last tiles split their K blocks among all
// workers (0: every tile data parallel). The reference's GemmPlan leaves this choice to
// cuBLASLt's heuristic (src/ops/gemm/plan/implementation.inc:13-60). Measured on B200
// (strict FP32, GEMM phase):
//  * one wave or more whose last wave leaves more than a tenth of the workers idle: the last
//    one or two waves' worth of tiles are shared (4096^3: 554 us against 678 us whole);
//  * tiles for at most 60% of the workers: all tiles are shared (512 x 512 x 65536: 180 us
//    against 1196-2193 us whole);
//  * tiles for 60-100% of the workers stay whole: 2048^3 took 87.7 us whole and 100.9 us
//    shared. Workers at staggered K offsets lose the L2 reuse that tiles moving through K in
//    lockstep get, and the fix-up pass costs more than the idle tenth of the SMs;
//  * every worker needs at least kMinSkBlocks K blocks: shorter shares spend more on filling
//    the pipeline and on the fix-up than they save.
constexpr int kMinSkBlocks = 8;

long long streamk_tiles(long long tiles, int workers, int kb) {
    if (workers <= 1 || tiles <= 0 || kb <= 0) return 0;
    if (tiles < workers && tiles * 10 > static_cast<long long>(workers) * 6) return 0;
    const long long waves = (tiles + workers - 1) / workers;
    if (tiles * 10 >= waves * workers * 9) return 0;
    const long long full = tiles / workers;
    const long long sk = full >= 1 ? tiles - (full - 1) * workers : tiles;
    if (sk * kb < static_cast<long long>(kMinSkBlocks) * workers) return 0;
    return sk;
}

// Most workers that share one stream-K tile.
int streamk_split(long long sk_tiles, int kb, int workers) {
    const long long iters = sk_tiles * kb;
    int most = 1;
    for (long long r = 0; r < sk_tiles; ++r)
        most = std::max(most, tc_sk_owner((r + 1) * kb - 1, iters, workers) - tc_sk_owner(r * kb, iters, workers) + 1);
    return most;
}

long long tile_count(const mfb_gemm_desc& d, const TcEntry& e, int n_cols, int batch) {
    const int rows = e.pair ? 2 * kTcBM : kTcBM;
    return static_cast<long long>(batch) * ((d.m + rows - 1) / rows) * ((n_cols + e.bn - 1) / e.bn);
}

int kb_count(const mfb_gemm_desc& d, const TcEntry& e) { return (d.k + kBK * e.kslabs - 1) / (kBK * e.kslabs); }

}  // namespace

// ------------------------------------------------------------------------------------
// Configuration choice
// ------------------------------------------------------------------------------------
int tc_candidates(const mfb_gemm_desc& d, TcConfig* out, int max_out, int batch) {
    const int planes = d.precision == MFB_PRECISION_TF32 ? 1 : 2;
    const int a_mn = d.trans_a ? 1 : 0;
    const int b_mn = d.trans_b ? 0 : 1;
    int count = 0;
    const TcEntry* t = kernel_table(&count);
    int dev = 0;
    cudaGetDevice(&dev);
    const int sms = sm_count(dev);
    // Estimated rate of each admissible kernel, as or without a stream-K launch: the tile
    // shape's per-SM rate (measured order: SM-pair 256 x 256 tiles, which halve B's
    // shared-memory traffic per FLOP, then 128 x 256, 128 x 128, 128 x 64) times the share of
    // workers that stay busy (whole waves of tiles, or ~90% with a stream-K share, the
    // fix-up included). mfb_plan_tune measures every candidate instead.
    struct Scored {
        TcConfig c;
        double score;
    };
    Scored all[32];
    int n_all = 0;
    for (int i = 0; i < count && n_all < 31; ++i) {
        const TcEntry& e = t[i];
        if (e.planes != planes || e.a_mn != a_mn || e.b_mn != b_mn) continue;
        const double rate = e.pair ? 1.0 : e.bn >= 256 ? 0.93 : e.bn >= 128 ? 0.8 : 0.6;
        const int workers = std::max(1, e.pair ? sms / 2 : sms);
        const long long tiles = tile_count(d, e, d.n, batch);
        const long long waves = (tiles + workers - 1) / workers;
        const double busy = waves > 0 ? static_cast<double>(tiles) / static_cast<double>(waves * workers) : 0.0;
        TcConfig c;
        c.bn = e.bn;
        c.stages = e.stages;
        c.planes = planes;
        c.a_mn = a_mn;
        c.b_mn = b_mn;
        c.pair = e.pair;
        c.stream_k = 0;
        all[n_all++] = Scored{c, rate * busy};
        if (streamk_tiles(tiles, workers, kb_count(d, e)) > 0) {
            c.stream_k = 1;
            all[n_all++] = Scored{c, rate * std::max(busy, 0.9)};
        }
    }
    std::stable_sort(all, all + n_all, [](const Scored& x, const Scored& y) { return x.score > y.score; });
    int n_out = 0;
    for (int i = 0; i < n_all && n_out < max_out; ++i) out[n_out++] = all[i].c;
    return n_out;
}

mfb_status_t tc_schedule(const mfb_gemm_desc& d, const TcConfig& cfg, int dev, int sm_limit, int batch,
                         int n_cols, TcSchedule* out) {
    const TcEntry* e = find_kernel(cfg);
    if (!e) return fail(MFB_EUNSUPPORTED, "no tcgen05 kernel for this tile configuration");
    TcSchedule sc;
    sc.tiles = tile_count(d, *e, n_cols, batch);
    sc.kb = kb_count(d, *e);
    MFB_TRY(worker_count(e, dev, sm_limit, &sc.workers));
    sc.sk_tiles = cfg.stream_k ? static_cast<int>(streamk_tiles(sc.tiles, sc.workers, sc.kb)) : 0;
    if (sc.sk_tiles > 0) {
        sc.split = streamk_split(sc.sk_tiles, sc.kb, sc.workers);
        sc.partial_bytes = 2ull * static_cast<size_t>(sc.workers) * static_cast<size_t>(e->pair ? 2 * kTcBM : kTcBM) *
                           static_cast<size_t>(e->bn) * 4u;
    }
    *out = sc;
    return MFB_OK;
}

size_t tc_workspace_bytes_for(const mfb_gemm_desc& d, const TcConfig& cfg, int batch) {
    size_t bytes = round_up(static_cast<long long>(tc_workspace_bytes(d, batch)), 256);
    int dev = 0;
    cudaGetDevice(&dev);
    TcSchedule sc;
    if (cfg.stream_k) {
        if (tc_schedule(d, cfg, dev, 0, batch, d.n, &sc) == MFB_OK)
            bytes += sc.partial_bytes;
        else
            clear_error();  // sized without a stream-K share; the launch then runs data parallel
    }
    return bytes;
}

size_t tc_workspace_bytes(const mfb_gemm_desc& d, int batch) {
    size_t bytes = 0;
    for (int which = 0; which < 2; ++which) {
        int rows, cols;
        long long ld;
        stored_dims(d, which == 0, &rows, &cols, &ld);
        (void)ld;
        // TF32: one round-to-nearest plane per operand; strict: hi and lo planes.
        bytes += (d.precision == MFB_PRECISION_TF32 ? 1 : 2) * plane_floats(rows, cols) * 4 *
                 static_cast<size_t>(std::max(1, batch));
    }
    return bytes;
}

mfb_status_t scale_output(const mfb_gemm_desc& d, cudaStream_t stream, float* c, const float* bias) {
    const long long total = static_cast<long long>(d.m) * d.n;
    if (total == 0) return MFB_OK;
    const int blocks = static_cast<int>(std::min<long long>((total + 255) / 256, static_cast<long long>(current_sm_count()) * 16));
    scale_epilogue_kernel<<<blocks, 256, 0, stream>>>(c, d.ldc, d.m, d.n, d.beta, bias, d.epilogue);
    MFB_CUDA_TRY(cudaGetLastError(), "scale/epilogue launch");
    return MFB_OK;
}

mfb_status_t tc_gemm(const mfb_gemm_desc& d, const TcConfig& cfg, cudaStream_t stream, const float* a,
                     const float* b, float* c, const float* bias, void* workspace, size_t workspace_bytes,
                     int phases, int sm_limit, const TcBatch& batch, const TcPrologue& prologue,
                     const TcColumns& cols) {
    const TcEntry* e = find_kernel(cfg);
    if (!e) return fail(MFB_EUNSUPPORTED, "no tcgen05 kernel for this tile configuration");
    const int nb = batch.count;
    if (nb < 1 || nb > 65535) return fail(MFB_EINVAL, "batch count must be in [1, 65535]");
    const bool run_prepass = (phases & kPhasePrepare) != 0;
    const bool run_gemm = (phases & kPhaseMultiply) != 0;
    const int n0 = cols.n0, n1 = cols.n1 < 0 ? d.n : cols.n1;
    const bool col_range = n0 != 0 || n1 != d.n || cols.b_src != nullptr;
    if (col_range && (d.trans_b || nb != 1 || n0 < 0 || n0 % 32 != 0 || n1 <= n0 || n1 > d.n ||
                      (n1 != d.n && n1 % 32 != 0)))
        return fail(MFB_EINVAL,
                    "column range needs a non-transposed B, one GEMM and 0 <= n0 < n1 <= n, n0 and n1 (unless n) "
                    "multiples of 32");

    // --- operand preparation: hi/lo planes (strict) or one rounded plane (TF32), laid out
    // [plane][batch entry][rows][cols rounded up to 4]. In the prepare-only phase a null
    // operand pointer skips that operand. ---
    PreparedOperand ops[2];
    SplitJob jobs[2] = {};
    size_t used = 0;
    char* ws = static_cast<char*>(workspace);
    if (prologue.shared_planes) {
        int ra, ca, rb, cb;
        long long la, lb;
        stored_dims(d, true, &ra, &ca, &la);
        stored_dims(d, false, &rb, &cb, &lb);
        if (a != b || la != lb || ra != rb || ca != cb || prologue.a_col_shift != prologue.b_col_shift ||
            cols.b_src != nullptr)
            return fail(MFB_EINVAL, "shared operand planes need A and B to be the same stored matrix");
    }
    for (int which = 0; which < 2; ++which) {
        PreparedOperand& op = ops[which];
        if (which == 1 && prologue.shared_planes) {
            op = ops[0];  // B reads A's planes
            break;
        }
        long long ld;
        stored_dims(d, which == 0, &op.rows, &op.cols, &ld);
        const float* src = which == 0 ? a : b;
        const long long src_batch = which == 0 ? batch.stride_a : batch.stride_b;
        const float* shift = which == 0 ? prologue.a_col_shift : prologue.b_col_shift;
        const long long ldp = round_up(op.cols, 4);
        const size_t pf = plane_floats(op.rows, op.cols);
        const size_t need = pf * 4 * static_cast<size_t>(cfg.planes) * static_cast<size_t>(nb);
        if (used + need > workspace_bytes || ws == nullptr)
            return fail(MFB_EINVAL, "workspace too small for the tcgen05 operand planes");
        float* hi = reinterpret_cast<float*>(ws + used);
        float* lo = cfg.planes == 2 ? hi + pf * nb : nullptr;
        used += need;
        const long long total_groups = static_cast<long long>(op.rows) * (ldp / 4);
        const int blocks = static_cast<int>(
            std::min<long long>((total_groups + 255) / 256, std::max(1LL, static_cast<long long>(current_sm_count()) * 8 / nb)));
        if (which == 1 && cols.b_src != nullptr) {
            // columns [n0, n1) of B from a separate matrix, into the same columns of the planes
            const bool vec_c = cols.b_ld % 4 == 0 && aligned16(cols.b_src);
            if (run_prepass)
                jobs[1] = SplitJob{cols.b_src, cols.b_ld, op.rows, n1 - n0, hi + n0, lo ? lo + n0 : nullptr, ldp,
                                   vec_c ? 1 : 0, 0, static_cast<long long>(pf), nullptr, blocks,
                                   round_up(static_cast<long long>(n1 - n0), 4)};
        } else {
            const bool vec = ld % 4 == 0 && src_batch % 4 == 0 && aligned16(src);
            if (run_prepass && src != nullptr)
                jobs[which] = SplitJob{src, ld, op.rows, op.cols, hi, lo, ldp, vec ? 1 : 0, src_batch,
                                       static_cast<long long>(pf), shift, blocks, ldp};
        }
        op.base = hi;
        op.ld = ldp;
        op.plane_stride = cfg.planes == 2 ? static_cast<long long>(pf) * nb : 0;
        op.batch_stride = static_cast<long long>(pf);
        op.needs_prepass = true;
    }
    const bool prepass_launched = jobs[0].blocks + jobs[1].blocks > 0;
    if (prepass_launched) {
        if (jobs[0].blocks == 0) std::swap(jobs[0], jobs[1]);  // a lone B job runs as the first
        split_tf32_kernel<<<dim3(jobs[0].blocks + jobs[1].blocks, nb), 256, 0, stream>>>(jobs[0], jobs[1]);
        MFB_CUDA_TRY(cudaGetLastError(), "split/pack prepass launch");
    }
    if (!run_gemm) return MFB_OK;

    // --- TMA descriptors ---
    CUtensorMap map_a, map_b;
    {
        const PreparedOperand& A = ops[0];
        // K-major A: box 32 (K) x 128 (M); MN-major A: box 32 (M) x 32 (K).
        MFB_TRY(encode_operand(&map_a, A.base, A.rows, A.cols, A.ld, cfg.planes, A.plane_stride, 32,
                               cfg.a_mn ? 32 : kTcBM, cfg.a_mn != 0, nb, A.batch_stride));
        const PreparedOperand& B = ops[1];
        // K-major B: box of the tile's columns, half of them per CTA on SM pairs; MN-major B: 32 x 32.
        const int b_rows = cfg.b_mn ? 32 : (e->pair ? cfg.bn / 2 : cfg.bn);
        MFB_TRY(encode_operand(&map_b, B.base, B.rows, B.cols, B.ld, cfg.planes, B.plane_stride, 32, b_rows,
                               cfg.b_mn != 0, nb, B.batch_stride));
    }

    GemmTcParams p{};
    p.m = d.m;
    p.n = n1;  // the launch's last output column + 1
    p.k = d.k;
    p.num_kb = (d.k + kBK * e->kslabs - 1) / (kBK * e->kslabs);
    const int tile_rows = cfg.pair ? 2 * kTcBM : kTcBM;
    p.tiles_m = (d.m + tile_rows - 1) / tile_rows;
    p.tiles_n = (n1 - n0 + cfg.bn - 1) / cfg.bn;
    p.n_base = n0;
    p.batch = nb;
    p.c_batch_stride = batch.stride_c;
    p.group_m = 16;
    p.c = c;
    p.ldc = d.ldc;
    p.alpha = d.alpha;
    p.beta = d.beta;
    p.bias = bias;
    p.epilogue = d.epilogue;
    p.c_vec4 = (aligned16(c) && d.ldc % 4 == 0) ? 1 : 0;
    p.wait_limit_ns = wait_limit_ns();

    const long long tiles = static_cast<long long>(p.tiles_m) * p.tiles_n * nb;
    if (tiles > 0x7fffffffLL) return fail(MFB_EINVAL, "problem has too many output tiles");
    int dev = 0;
    cudaGetDevice(&dev);
    // Persistent: one CTA per SM (or SM pair), or fewer when the caller leaves SMs to a
    // concurrent collective. A stream-K launch keeps every worker; its partial slots follow
    // the operand planes in the workspace (column-range calls stay data parallel).
    TcConfig launch_cfg = cfg;
    if (col_range) launch_cfg.stream_k = 0;
    TcSchedule sc;
    MFB_TRY(tc_schedule(d, launch_cfg, dev, sm_limit, nb, n1 - n0, &sc));
    const size_t partial_off = static_cast<size_t>(round_up(static_cast<long long>(used), 256));
    if (sc.sk_tiles > 0 && partial_off + sc.partial_bytes <= workspace_bytes) {
        p.sk_tiles = sc.sk_tiles;
        p.partials = reinterpret_cast<float*>(ws + partial_off);
    } else {
        p.sk_tiles = 0;  // no room for the partial slots: every tile data parallel
        p.partials = nullptr;
    }
    const long long workers = p.sk_tiles > 0 ? sc.workers : std::min<long long>(tiles, sc.workers);
    MFB_TRY(set_kernel_attributes(e));
    void* args[] = {&map_a, &map_b, &p};
    // Right after this call's prepass the GEMM launches programmatically: its CTAs set up
    // (barriers, TMEM, descriptor prefetch) while the prepass drains, then wait for it.
    cudaLaunchAttribute pdl;
    pdl.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl.val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t lc{};
    cudaLaunchAttribute attr[2];
    lc.blockDim = dim3(e->threads);
    lc.dynamicSmemBytes = static_cast<size_t>(e->smem);
    lc.stream = stream;
    if (!e->pair) {
        lc.gridDim = dim3(static_cast<unsigned>(workers));
        lc.attrs = &pdl;
        lc.numAttrs = prepass_launched ? 1 : 0;
        MFB_CUDA_TRY(cudaLaunchKernelExC(&lc, e->fn, args), "tcgen05 GEMM launch");
    } else {
        // SM pairs: clusters of 2 CTAs, as many as can be co-resident (capped by the SM limit).
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        attr[1] = pdl;
        lc.gridDim = dim3(static_cast<unsigned>(2 * workers));
        lc.attrs = attr;
        lc.numAttrs = prepass_launched ? 2 : 1;
        MFB_CUDA_TRY(cudaLaunchKernelExC(&lc, e->fn, args), "tcgen05 pair GEMM launch");
    }
    if (p.sk_tiles == 0) return MFB_OK;
    // The fix-up of the shared tiles, launched programmatically behind the GEMM.
    int w = static_cast<int>(sc.workers);
    void* rargs[] = {&p, &w};
    cudaLaunchConfig_t rc{};
    const int per_tile = tile_rows * cfg.bn / 4;  // float4 groups of one tile, one per thread
    rc.gridDim = dim3(static_cast<unsigned>((per_tile + 255) / 256), static_cast<unsigned>(p.sk_tiles));
    rc.blockDim = dim3(256);
    rc.stream = stream;
    rc.attrs = &pdl;
    rc.numAttrs = 1;
    MFB_CUDA_TRY(cudaLaunchKernelExC(&rc, e->reduce, rargs), "stream-K fix-up launch");
    return MFB_OK;
}

}  // namespace mfb
