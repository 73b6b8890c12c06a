// The reference-side bodies of the Matrix-level GEMM API and of conv2d over libmfb.so's C ABI,
// compiled as a stand-alone C++17 program:
//   GemmPlan (include/matrix_pro/ops/gemm.hpp:36-62; body src/ops/gemm/plan/implementation.inc:5-152),
//   gemm_into / gemm with the bounded per-thread plan cache (convenience.inc:5-27, cache.inc:8-50),
//   conv2d (include/matrix_pro/nn/conv.hpp:16-17; body src/nn/conv.cu:110-163).
// Matrix and Tensor are small stand-ins for the reference's containers
// (include/matrix_pro/core/matrix.hpp, tensor.hpp): host data with a lazily uploaded device
// mirror, mark_host_stale() / download() as there. compute_stream() is a per-thread, per-device
// stream like the reference's. main() runs the reference's known answers of
// tests/unit/test_gemm_plan.cpp:14-88 and tests/unit/test_conv.cpp:31-67.
// Exit code 0 = all checks passed.
#include "mfb.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <future>
#include <list>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <tuple>
#include <utility>
#include <vector>

namespace matrix_pro {

// Same names and bases as include/matrix_pro/core/errors.hpp.
class MatrixProError : public std::runtime_error {
public:
    using std::runtime_error::runtime_error;
};
class InvalidArgumentError : public MatrixProError {
public:
    using MatrixProError::MatrixProError;
};
class ShapeMismatchError : public MatrixProError {
public:
    using MatrixProError::MatrixProError;
};
class CudaError : public MatrixProError {
public:
    using MatrixProError::MatrixProError;
};

namespace {
void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

// mfb_status_t -> the reference's exception classes.
void check_mfb(mfb_status_t st, const char* what) {
    if (st == MFB_OK) return;
    const std::string msg = std::string(what) + ": " + mfb_last_error();
    if (st == MFB_EINVAL) throw InvalidArgumentError(msg);
    if (st == MFB_ESHAPE) throw ShapeMismatchError(msg);
    throw CudaError(msg);
}

int current_device() {
    int d = 0;
    check_cuda(cudaGetDevice(&d), "cudaGetDevice");
    return d;
}

// One compute stream per thread and device, created on first use.
cudaStream_t compute_stream() {
    thread_local std::vector<cudaStream_t> streams;
    const int d = current_device();
    if (static_cast<int>(streams.size()) <= d) streams.resize(d + 1, nullptr);
    if (!streams[d]) check_cuda(cudaStreamCreateWithFlags(&streams[d], cudaStreamNonBlocking), "compute stream");
    return streams[d];
}

void synchronize() { check_cuda(cudaStreamSynchronize(compute_stream()), "synchronize"); }

mfb_stream_t mfb_stream(cudaStream_t s) { return reinterpret_cast<mfb_stream_t>(s); }

int checked_dim(std::size_t value) {
    if (value > static_cast<std::size_t>(INT_MAX))
        throw InvalidArgumentError("GEMM dimension exceeds the 32-bit backend limit");
    return static_cast<int>(value);
}

void require_not_capturing(cudaStream_t stream) {
    cudaStreamCaptureStatus status;
    check_cuda(cudaStreamIsCapturing(stream, &status), "GEMM capture query");
    if (status != cudaStreamCaptureStatusNone)
        throw InvalidArgumentError("Construct/tune GEMM plans before CUDA Graph capture");
}
}  // namespace

// ------------------------------------------------------------------ containers (stand-ins)
class DeviceMirror {
public:
    DeviceMirror() = default;
    explicit DeviceMirror(std::vector<float> host) : host_(std::move(host)) {}
    DeviceMirror(DeviceMirror&& o) noexcept { *this = std::move(o); }
    DeviceMirror& operator=(DeviceMirror&& o) noexcept {
        std::swap(host_, o.host_);
        std::swap(dev_, o.dev_);
        std::swap(dev_current_, o.dev_current_);
        std::swap(host_current_, o.host_current_);
        return *this;
    }
    ~DeviceMirror() {
        if (dev_) cudaFree(dev_);
    }
    std::size_t size() const { return host_.size(); }
    const float* device_data() const { return const_cast<DeviceMirror*>(this)->device_data(); }
    float* device_data() {
        if (host_.empty()) return nullptr;
        if (!dev_) check_cuda(cudaMalloc(&dev_, host_.size() * 4), "device allocation");
        if (!dev_current_) upload();
        return dev_;
    }
    void upload() {
        if (host_.empty()) return;
        if (!dev_) check_cuda(cudaMalloc(&dev_, host_.size() * 4), "device allocation");
        check_cuda(cudaMemcpy(dev_, host_.data(), host_.size() * 4, cudaMemcpyHostToDevice), "upload");
        dev_current_ = true;
    }
    void mark_host_stale() {
        host_current_ = false;
        dev_current_ = true;
    }
    bool host_current() const { return host_current_; }
    void download() {
        if (host_current_ || !dev_) return;
        check_cuda(cudaStreamSynchronize(compute_stream()), "download sync");
        check_cuda(cudaMemcpy(host_.data(), dev_, host_.size() * 4, cudaMemcpyDeviceToHost), "download");
        host_current_ = true;
    }
    std::vector<float>& data() { return host_; }
    const std::vector<float>& data() const { return host_; }

private:
    std::vector<float> host_;
    float* dev_ = nullptr;
    bool dev_current_ = false;
    bool host_current_ = true;
};

class Matrix : public DeviceMirror {
public:
    Matrix(std::size_t rows, std::size_t cols) : DeviceMirror(std::vector<float>(rows * cols, 0.0f)), r_(rows), c_(cols) {}
    Matrix(std::size_t rows, std::size_t cols, std::vector<float> v) : DeviceMirror(std::move(v)), r_(rows), c_(cols) {}
    static Matrix ones(std::size_t r, std::size_t c) { return Matrix(r, c, std::vector<float>(r * c, 1.0f)); }
    static Matrix identity(std::size_t n) {
        Matrix m(n, n);
        for (std::size_t i = 0; i < n; ++i) m.data()[i * n + i] = 1.0f;
        return m;
    }
    static Matrix random(std::size_t r, std::size_t c, unsigned seed) {
        Matrix m(r, c);
        for (auto& v : m.data()) {
            seed = seed * 1664525u + 1013904223u;
            v = static_cast<float>((seed >> 8) & 0xFFFF) / 65536.0f;
        }
        return m;
    }
    std::size_t rows() const { return r_; }
    std::size_t cols() const { return c_; }
    bool empty() const { return size() == 0; }
    float at(std::size_t i, std::size_t j) const { return data()[i * c_ + j]; }

private:
    std::size_t r_, c_;
};

class Tensor : public DeviceMirror {
public:
    Tensor(std::vector<std::size_t> shape, std::vector<float> v) : DeviceMirror(std::move(v)), shape_(std::move(shape)) {}
    explicit Tensor(std::vector<std::size_t> shape) : DeviceMirror(std::vector<float>(count(shape), 0.0f)), shape_(shape) {}
    const std::vector<std::size_t>& shape() const { return shape_; }
    std::size_t rank() const { return shape_.size(); }

private:
    static std::size_t count(const std::vector<std::size_t>& s) {
        std::size_t n = 1;
        for (auto d : s) n *= d;
        return n;
    }
    std::vector<std::size_t> shape_;
};

// ------------------------------------------------------------------ GEMM API
enum class GemmPrecision { fp32, tf32 };
enum class GemmEpilogue { none, bias, bias_relu, bias_gelu };
struct GemmOptions {
    bool transpose_left = false;
    bool transpose_right = false;
    GemmPrecision precision = GemmPrecision::fp32;
    GemmEpilogue epilogue = GemmEpilogue::none;
    std::size_t workspace_limit_bytes = 64u << 20;
};
struct GemmTuningResult {
    int candidates_tested = 0;
    float selected_ms = 0;
};

class GemmPlan {
public:
    GemmPlan(std::size_t m, std::size_t n, std::size_t k, GemmOptions options = {});
    ~GemmPlan();
    GemmPlan(GemmPlan&&) noexcept;
    GemmPlan& operator=(GemmPlan&&) noexcept;
    void execute(const Matrix& left, const Matrix& right, Matrix& output, float alpha = 1, float beta = 0,
                 const Matrix* bias = nullptr);
    GemmTuningResult tune(const Matrix& left, const Matrix& right, const Matrix& output, float alpha = 1,
                          float beta = 0, const Matrix* bias = nullptr, int repeats = 5);
    std::size_t rows() const noexcept;
    std::size_t cols() const noexcept;
    std::size_t inner() const noexcept;
    int candidate_count() const noexcept;
    bool uses_cublaslt() const noexcept;

private:
    struct Impl;
    std::unique_ptr<Impl> impl_;
};

// GemmPlan::Impl keeps the reference's validation (implementation.inc:88-110) and holds an
// mfb_plan_t where the reference holds cuBLASLt descriptors and heuristics.
struct GemmPlan::Impl {
    int m, n, k, device;
    GemmOptions options;
    cudaStream_t stream;
    std::thread::id owner = std::this_thread::get_id();
    mfb_plan_t plan = nullptr;

    Impl(std::size_t rows, std::size_t cols, std::size_t inner, GemmOptions o)
        : m(checked_dim(rows)), n(checked_dim(cols)), k(checked_dim(inner)), device(current_device()), options(o),
          stream(compute_stream()) {
        require_not_capturing(stream);
        mfb_gemm_desc d{};
        d.m = m;
        d.n = n;
        d.k = k;
        d.lda = o.transpose_left ? std::max(m, 1) : std::max(k, 1);   // contiguous Matrix operands
        d.ldb = o.transpose_right ? std::max(k, 1) : std::max(n, 1);
        d.ldc = std::max(n, 1);
        d.alpha = 1.0f;
        d.beta = 0.0f;
        d.precision = o.precision == GemmPrecision::tf32 ? MFB_PRECISION_TF32 : MFB_PRECISION_FP32;
        d.trans_a = o.transpose_left ? 1 : 0;
        d.trans_b = o.transpose_right ? 1 : 0;
        d.epilogue = static_cast<int>(o.epilogue);
        check_mfb(mfb_plan_create(device, &d, &plan), "GemmPlan");
    }
    ~Impl() { mfb_plan_destroy(plan); }

    void validate(const Matrix& left, const Matrix& right, const Matrix& output, const Matrix* bias) const {
        if (std::this_thread::get_id() != owner || current_device() != device || compute_stream() != stream)
            throw InvalidArgumentError("GEMM plan must execute on its creating thread, device and stream");
        if (left.rows() != static_cast<std::size_t>(options.transpose_left ? k : m) ||
            left.cols() != static_cast<std::size_t>(options.transpose_left ? m : k) ||
            right.rows() != static_cast<std::size_t>(options.transpose_right ? n : k) ||
            right.cols() != static_cast<std::size_t>(options.transpose_right ? k : n) ||
            output.rows() != static_cast<std::size_t>(m) || output.cols() != static_cast<std::size_t>(n))
            throw ShapeMismatchError("GEMM plan operand shape mismatch");
        if (!output.empty() && (output.device_data() == left.device_data() || output.device_data() == right.device_data()))
            throw InvalidArgumentError("GEMM output cannot alias an input");
        if (options.epilogue != GemmEpilogue::none) {
            if (!bias || bias->size() != static_cast<std::size_t>(n))
                throw ShapeMismatchError("GEMM bias length must equal N");
            if (!output.empty() && output.device_data() == bias->device_data())
                throw InvalidArgumentError("GEMM output cannot alias bias");
        }
    }

    void run_ptr(const float* left, const float* right, float* output, float alpha, float beta, const float* bias) {
        check_mfb(mfb_plan_execute(plan, mfb_stream(stream), left, right, output, alpha, beta, bias), "GEMM");
    }
};

GemmPlan::GemmPlan(std::size_t m, std::size_t n, std::size_t k, GemmOptions options)
    : impl_(std::make_unique<Impl>(m, n, k, options)) {}
GemmPlan::~GemmPlan() = default;
GemmPlan::GemmPlan(GemmPlan&&) noexcept = default;
GemmPlan& GemmPlan::operator=(GemmPlan&&) noexcept = default;

void GemmPlan::execute(const Matrix& left, const Matrix& right, Matrix& output, float alpha, float beta,
                       const Matrix* bias) {
    if (!impl_) throw InvalidArgumentError("Cannot execute a moved-from GEMM plan");
    impl_->validate(left, right, output, bias);
    impl_->run_ptr(left.device_data(), right.device_data(), output.device_data(), alpha, beta,
                   bias ? bias->device_data() : nullptr);
    output.mark_host_stale();
}

GemmTuningResult GemmPlan::tune(const Matrix& left, const Matrix& right, const Matrix& output, float, float,
                                const Matrix* bias, int repeats) {
    if (!impl_) throw InvalidArgumentError("Cannot tune a moved-from GEMM plan");
    impl_->validate(left, right, output, bias);
    require_not_capturing(impl_->stream);
    Matrix scratch(output.rows(), output.cols());  // output and beta's input stay unchanged
    GemmTuningResult r;
    check_mfb(mfb_plan_tune(impl_->plan, mfb_stream(impl_->stream), left.device_data(), right.device_data(),
                            scratch.device_data(), repeats, &r.candidates_tested, &r.selected_ms),
              "GEMM tune");
    return r;
}

std::size_t GemmPlan::rows() const noexcept { return impl_ ? impl_->m : 0; }
std::size_t GemmPlan::cols() const noexcept { return impl_ ? impl_->n : 0; }
std::size_t GemmPlan::inner() const noexcept { return impl_ ? impl_->k : 0; }
int GemmPlan::candidate_count() const noexcept {
    mfb_plan_info info{};
    return impl_ && mfb_plan_info_get(impl_->plan, &info) == MFB_OK ? info.candidates : 0;
}
// The reference reports whether cuBLASLt serves the plan; here: whether the tcgen05 GEMM does.
bool GemmPlan::uses_cublaslt() const noexcept {
    mfb_plan_info info{};
    return impl_ && mfb_plan_info_get(impl_->plan, &info) == MFB_OK && info.path == 0;
}

namespace {
// Bounded per-thread plan cache keyed by device, stream, shape and options (cache.inc:8-50).
GemmPlan& cached(std::size_t m, std::size_t n, std::size_t k, const GemmOptions& o) {
    using Key = std::tuple<int, cudaStream_t, std::size_t, std::size_t, std::size_t, bool, bool, int, int>;
    thread_local std::list<std::pair<Key, GemmPlan>> cache;
    const Key key{current_device(), compute_stream(), m, n, k, o.transpose_left, o.transpose_right,
                  static_cast<int>(o.precision), static_cast<int>(o.epilogue)};
    for (auto it = cache.begin(); it != cache.end(); ++it) {
        if (it->first == key) {
            cache.splice(cache.begin(), cache, it);
            return cache.front().second;
        }
    }
    if (cache.size() >= 128) cache.pop_back();
    cache.emplace_front(key, GemmPlan(m, n, k, o));
    return cache.front().second;
}
}  // namespace

void gemm_into(const Matrix& left, const Matrix& right, Matrix& output, GemmOptions o = {}, float alpha = 1,
               float beta = 0, const Matrix* bias = nullptr) {
    const auto m = o.transpose_left ? left.cols() : left.rows(), k = o.transpose_left ? left.rows() : left.cols();
    const auto n = o.transpose_right ? right.rows() : right.cols();
    if (k != (o.transpose_right ? right.cols() : right.rows())) throw ShapeMismatchError("GEMM inner dimension mismatch");
    cached(m, n, k, o).execute(left, right, output, alpha, beta, bias);
}

Matrix gemm(const Matrix& left, const Matrix& right, GemmOptions o = {}, float alpha = 1,
            const Matrix* bias = nullptr) {
    const auto m = o.transpose_left ? left.cols() : left.rows(), n = o.transpose_right ? right.rows() : right.cols();
    checked_dim(m);
    checked_dim(n);
    Matrix output(m, n);
    gemm_into(left, right, output, o, alpha, 0, bias);
    return output;
}

// ------------------------------------------------------------------ conv2d (src/nn/conv.cu:110-163)
Tensor conv2d(const Tensor& input, const Tensor& weights, const Tensor& bias, std::size_t stride = 1,
              std::size_t padding = 0) {
    if (input.rank() != 4) throw InvalidArgumentError("conv2d expects an NCHW input");
    if (weights.rank() != 4 || bias.rank() != 1) throw InvalidArgumentError("conv2d expects weights [K,C,R,S] and bias [K]");
    const auto& x = input.shape();
    const auto& w = weights.shape();
    if (w[1] != x[1] || bias.shape()[0] != w[0] || stride == 0) throw ShapeMismatchError("conv2d channel or stride mismatch");
    if (x[2] + 2 * padding < w[2] || x[3] + 2 * padding < w[3])
        throw ShapeMismatchError("conv2d kernel is larger than padded input");
    const std::size_t oh = (x[2] + 2 * padding - w[2]) / stride + 1;
    const std::size_t ow = (x[3] + 2 * padding - w[3]) / stride + 1;
    Tensor output({x[0], w[0], oh, ow});
    check_mfb(mfb_conv2d_fwd(current_device(), mfb_stream(compute_stream()), int(x[0]), int(x[1]), int(x[2]), int(x[3]),
                             int(w[0]), int(w[2]), int(w[3]), int(stride), int(padding), input.device_data(),
                             weights.device_data(), bias.device_data(), output.device_data(), MFB_PRECISION_FP32),
              "conv2d");
    output.mark_host_stale();
    return output;
}

}  // namespace matrix_pro

// ====================================================================== known answers
using namespace matrix_pro;

namespace {
int failures = 0;
int checks = 0;
void check(bool ok, const char* what) {
    ++checks;
    if (!ok) {
        ++failures;
        std::printf("[FAIL] %s\n", what);
    }
}
void check_near(double v, double ref, double tol, const char* what) { check(std::fabs(v - ref) <= tol, what); }
template <class E, class F>
void check_throws(F f, const char* what) {
    bool ok = false;
    try {
        f();
    } catch (const E&) {
        ok = true;
    } catch (...) {
    }
    check(ok, what);
}
const float& at_nchw(const Tensor& t, std::size_t n, std::size_t c, std::size_t h, std::size_t w) {
    const std::size_t C = t.shape()[1], H = t.shape()[2], W = t.shape()[3];
    return t.data()[((n * C + c) * H + h) * W + w];
}
}  // namespace

int main() {
    try {
        // --- test_gemm_plan.cpp:14-34: transposes, scaling, accumulation, fused epilogues
        for (bool ta : {false, true})
            for (bool tb : {false, true})
                for (int ep = 0; ep < 4; ++ep) {
                    const int m = 7, n = 9, k = 5;
                    std::vector<float> av(m * k), bv(k * n), biasv(n);
                    for (size_t i = 0; i < av.size(); ++i) av[i] = (static_cast<int>(i % 11) - 5) * 0.17f;
                    for (size_t i = 0; i < bv.size(); ++i) bv[i] = (static_cast<int>(i % 7) - 3) * 0.23f;
                    for (int i = 0; i < n; ++i) biasv[i] = (i - 4) * 0.11f;
                    Matrix a(ta ? k : m, ta ? m : k, av), b(tb ? n : k, tb ? k : n, bv), bias(1, n, biasv);
                    Matrix c = Matrix::ones(m, n);
                    GemmOptions o;
                    o.transpose_left = ta;
                    o.transpose_right = tb;
                    o.epilogue = static_cast<GemmEpilogue>(ep);
                    GemmPlan p(m, n, k, o);
                    p.execute(a, b, c, 0.7f, -0.3f, ep ? &bias : nullptr);
                    check(!c.host_current(), "execute invalidates host mirror");
                    c.download();
                    for (int i = 0; i < m; ++i)
                        for (int j = 0; j < n; ++j) {
                            double dot = 0;
                            for (int t = 0; t < k; ++t)
                                dot += static_cast<double>(av[ta ? t * m + i : i * k + t]) * bv[tb ? j * k + t : t * n + j];
                            double ref = 0.7f * dot - 0.3f;
                            if (ep) ref += biasv[j];
                            if (ep == 2) ref = std::max(0.0, ref);
                            if (ep == 3) ref = 0.5 * ref * (1 + std::tanh(0.7978845608 * (ref + 0.044715 * ref * ref * ref)));
                            check_near(c.at(i, j), ref, 3e-5, "GEMM agrees with independent double dot product");
                        }
                }
        // --- :36-50: empty inner dimension, alias rejection and validation
        {
            Matrix a(3, 0), b(0, 4), c = Matrix::ones(3, 4), bias = Matrix::ones(1, 4);
            GemmOptions o;
            o.epilogue = GemmEpilogue::bias_relu;
            GemmPlan empty(3, 4, 0, o);
            empty.execute(a, b, c, 1, -2, &bias);
            c.download();
            for (float x : c.data()) check_near(x, 0, 0, "empty K applies beta and epilogue");
            empty.execute(a, b, c, 1, 0, &bias);
            c.download();
            for (float x : c.data()) check_near(x, 1, 0, "empty K zero beta");
            Matrix square = Matrix::identity(3);
            GemmPlan p(3, 3, 3);
            check_throws<InvalidArgumentError>([&] { p.execute(square, square, square); }, "reject output alias");
            check_throws<ShapeMismatchError>([&] { p.execute(square, b, c); }, "reject operand mismatch");
            check_throws<InvalidArgumentError>([] { GemmPlan huge(static_cast<size_t>(INT_MAX) + 1, 1, 1); },
                                               "reject int overflow before allocation");
            GemmPlan moved = std::move(p);
            check_throws<InvalidArgumentError>([&] { p.execute(square, square, square); }, "reject moved-from plan");
            Matrix out(3, 3);
            moved.execute(square, square, out);
            out.download();
            check(out.at(1, 1) == 1.0f && out.at(0, 1) == 0.0f, "the moved-to plan runs");
        }
        // --- :52-66: tuning keeps beta's input; a captured TF32 execute reads updated inputs
        {
            Matrix left = Matrix::random(128, 128, 17), right = Matrix::random(128, 128, 23);
            Matrix out = Matrix::ones(128, 128);
            GemmOptions fast;
            fast.precision = GemmPrecision::tf32;
            GemmPlan plan(128, 128, 128, fast);
            auto tuning = plan.tune(left, right, out, 1, 0.5f);
            check(tuning.candidates_tested > 0, "tuning measured candidates");
            out.download();
            for (float x : out.data()) check_near(x, 1, 0, "tuning leaves output unchanged");
            Matrix reference = gemm(left, right);
            reference.download();
            plan.execute(left, right, out);
            synchronize();
            cudaGraph_t graph = nullptr;
            cudaGraphExec_t exec = nullptr;
            check_cuda(cudaStreamBeginCapture(compute_stream(), cudaStreamCaptureModeThreadLocal), "begin capture");
            plan.execute(left, right, out);
            check_cuda(cudaStreamEndCapture(compute_stream(), &graph), "end capture");
            check_cuda(cudaGraphInstantiate(&exec, graph, 0), "instantiate");
            check_cuda(cudaGraphLaunch(exec, compute_stream()), "replay");
            out.mark_host_stale();
            out.download();
            for (size_t i = 0; i < out.size(); ++i)
                check_near(out.data()[i], reference.data()[i], 0.025, "TF32 graph agrees with FP32 reference");
            std::fill(right.data().begin(), right.data().end(), 0.0f);
            right.upload();
            check_cuda(cudaGraphLaunch(exec, compute_stream()), "replay");
            out.mark_host_stale();
            out.download();
            for (float x : out.data()) check_near(x, 0, 0, "graph reads updated input buffers");
            cudaGraphExecDestroy(exec);
            cudaGraphDestroy(graph);
        }
        // --- :68-80: vectors keep full FP32 input precision
        for (size_t inner : {size_t(127), size_t(2048)}) {
            Matrix vector = Matrix::random(1, inner, 91), weights = Matrix::random(inner, 127, 97);
            for (auto& v : vector.data()) v -= 0.5f;
            for (auto& v : weights.data()) v -= 0.5f;
            vector.upload();
            weights.upload();
            Matrix product = gemm(vector, weights);
            product.download();
            for (size_t j = 0; j < weights.cols(); ++j) {
                double ref = 0;
                for (size_t t = 0; t < weights.rows(); ++t)
                    ref += static_cast<double>(vector.data()[t]) * weights.data()[t * weights.cols() + j];
                check_near(product.at(0, j), ref, 2e-5, "long vector agrees with strict double-dot tolerance");
            }
        }
        // --- :81-88: the cached GEMM on two threads at once
        auto worker = [](float value) {
            Matrix x(256, 256, std::vector<float>(256 * 256, value)), y = Matrix::ones(256, 256), z(256, 256);
            for (int i = 0; i < 10; ++i) gemm_into(x, y, z);
            z.download();
            return z.at(127, 129);
        };
        auto f = std::async(std::launch::async, worker, 2.0f), g = std::async(std::launch::async, worker, -3.0f);
        check_near(f.get(), 512, 0.01, "thread one workspace isolated");
        check_near(g.get(), -768, 0.01, "thread two workspace isolated");

        // --- test_conv.cpp:31-67: conv2d forward, padding and stride
        {
            Tensor in2({1, 1, 2, 2}, {1.0f, 2.0f, 3.0f, 4.0f});
            Tensor k1({1, 1, 1, 1}, {1.0f});
            Tensor b0({1}, {0.0f});
            Tensor out = conv2d(in2, k1, b0);
            out.download();
            check(out.shape() == std::vector<std::size_t>{1, 1, 2, 2}, "identity conv keeps the input shape");
            check(std::fabs(at_nchw(out, 0, 0, 1, 1) - 4.0f) < 1e-5f, "an all-ones kernel reproduces the input");
            Tensor in3({1, 1, 3, 3}, {1.0f, 2.0f, 3.0f, 4.0f, 5.0f, 6.0f, 7.0f, 8.0f, 9.0f});
            Tensor k2({1, 1, 2, 2}, {1.0f, 1.0f, 1.0f, 1.0f});
            Tensor win = conv2d(in3, k2, b0);
            win.download();
            check(win.shape() == std::vector<std::size_t>{1, 1, 2, 2}, "2x2 kernel shrinks the output by k-1");
            check(std::fabs(at_nchw(win, 0, 0, 0, 0) - 12.0f) < 1e-4f, "top-left window sums to 12");
            check(std::fabs(at_nchw(win, 0, 0, 1, 1) - 28.0f) < 1e-4f, "bottom-right window sums to 28");
            Tensor biased = conv2d(in3, k2, Tensor({1}, {10.0f}));
            biased.download();
            check(std::fabs(at_nchw(biased, 0, 0, 0, 0) - 22.0f) < 1e-4f, "bias is added once per output element");
            Tensor padded = conv2d(in2, k1, b0, 1, 1);
            padded.download();
            check(padded.shape() == std::vector<std::size_t>{1, 1, 4, 4}, "padding 1 on a 1x1 kernel grows the output by 2*pad");
            Tensor in4({1, 1, 4, 4}, {1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16});
            Tensor stride2 = conv2d(in4, k1, b0, 2, 0);
            stride2.download();
            check(stride2.shape() == std::vector<std::size_t>{1, 1, 2, 2}, "stride 2 halves a 4x4 output");
            check(std::fabs(at_nchw(stride2, 0, 0, 0, 0) - 1.0f) < 1e-5f && std::fabs(at_nchw(stride2, 0, 0, 0, 1) - 3.0f) < 1e-5f &&
                      std::fabs(at_nchw(stride2, 0, 0, 1, 1) - 11.0f) < 1e-5f,
                  "stride 2 samples the top-left of each window");
            check_throws<ShapeMismatchError>([&] { conv2d(in3, Tensor({1, 2, 2, 2}), b0); }, "channel mismatch throws");
        }
    } catch (const std::exception& e) {
        std::printf("unexpected exception: %s\n", e.what());
        return 1;
    }
    std::printf("%d checks, %d failure(s)\n", checks, failures);
    return failures == 0 ? 0 : 1;
}
