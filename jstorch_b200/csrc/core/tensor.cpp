// tensor.cpp -- host core Tensor (see tensor.h).
#include "tensor.h"

#include <algorithm>
#include <atomic>
#include <numeric>
#include <sstream>
#include <stdexcept>

#include "../../../include/jstorch_gemm.h"
#include "core_kernels.h"

namespace jst {
namespace core {

namespace {
cudaStream_t g_stream = nullptr;  // legacy default stream, as the reference
std::atomic<uint64_t> g_randn_seed{42};

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
    }
}

void check_jst(int rc, const char* what) {
    if (rc != JST_OK) throw std::runtime_error(std::string(what) + ": " + jst_last_error());
}

int norm_axis(int axis, int nd) {
    if (axis < 0) axis += nd;
    if (axis < 0 || axis >= nd) throw std::runtime_error("Axis out of range");
    return axis;
}

// GEMM operand description of the last two dims of t.
struct Operand {
    const float* ptr;
    int trans;
    int64_t ld;
    int64_t bstride;
};

// Row-major -> trans 0; transposed view (unit stride along rows) -> trans 1.
bool describe(const Tensor& t, Operand* o) {
    const int nd = t.ndim();
    const int64_t rows = t.shape()[nd - 2], cols = t.shape()[nd - 1];
    const int64_t s0 = t.strides()[nd - 2], s1 = t.strides()[nd - 1];
    o->ptr = t.data();
    o->bstride = nd == 3 ? t.strides()[0] : 0;
    if (s1 == 1 && (rows <= 1 || s0 >= cols)) {
        o->trans = 0;
        o->ld = std::max<int64_t>(rows > 1 ? s0 : cols, 1);
        return true;
    }
    if (s0 == 1 && (cols <= 1 || s1 >= rows)) {
        o->trans = 1;
        o->ld = std::max<int64_t>(cols > 1 ? s1 : rows, 1);
        return true;
    }
    return false;
}

// C[b] = op(A[b]) op(B[b]) (+ bias) on the core stream.
void gemm(const Tensor& a_in, const Tensor& b_in, Tensor& c, int64_t batch, const Tensor* bias) {
    Tensor a = a_in, b = b_in;
    Operand oa, ob;
    if (!describe(a, &oa)) {
        a = a.contiguous();
        describe(a, &oa);
    }
    if (!describe(b, &ob)) {
        b = b.contiguous();
        describe(b, &ob);
    }
    const int nd = a.ndim();
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, (int)a.shape()[nd - 2], (int)b.shape()[b.ndim() - 1], (int)a.shape()[nd - 1], oa.ptr,
                       ob.ptr, c.data());
    d.transA = oa.trans;
    d.lda = oa.ld;
    d.strideA = oa.bstride;
    d.transB = ob.trans;
    d.ldb = ob.ld;
    d.strideB = ob.bstride;
    d.ldc = d.N;
    d.strideC = (int64_t)d.M * d.N;
    d.batch = (int)batch;
    Tensor bias_c;
    if (bias) {
        bias_c = bias->contiguous();
        d.bias = bias_c.data();
        d.epilogue = JST_EPI_BIAS;
    }
    d.stream = reinterpret_cast<jst_stream_t>(g_stream);
    check_jst(jst_gemm_ex(&d), "matmul");
}
}  // namespace

int64_t numel(const Shape& s) {
    return s.empty() ? 0 : std::accumulate(s.begin(), s.end(), int64_t(1), std::multiplies<int64_t>());
}

Shape contiguous_strides(const Shape& s) {
    Shape st(s.size());
    int64_t acc = 1;
    for (int i = (int)s.size() - 1; i >= 0; --i) {
        st[i] = acc;
        acc *= s[i];
    }
    return st;
}

std::string shape_str(const Shape& s) {
    std::ostringstream o;
    o << "[";
    for (size_t i = 0; i < s.size(); ++i) o << (i ? ", " : "") << s[i];
    o << "]";
    return o.str();
}

cudaStream_t core_stream() { return g_stream; }
void set_core_stream(cudaStream_t s) { g_stream = s; }

void clear_cache() { trim_all(); }

Tensor::Tensor(const Shape& shape) : shape_(shape), strides_(contiguous_strides(shape)) {
    for (auto d : shape)
        if (d < 0) throw std::runtime_error("negative dimension in " + shape_str(shape));
    block_ = device_alloc((size_t)numel(shape) * sizeof(float));
}

bool Tensor::is_contiguous() const {
    int64_t expected = 1;
    for (int i = ndim() - 1; i >= 0; --i) {
        if (shape_[i] != 1 && strides_[i] != expected) return false;
        expected *= shape_[i];
    }
    return true;
}

Tensor Tensor::from_buffer(const float* host, int64_t count, const Shape& shape) {
    if (numel(shape) != count) throw std::runtime_error("from_buffer: size mismatch");
    Tensor r(shape);
    // pinned, double-buffered staging (jst_copy_h2d); ready in core-stream order
    if (jst_copy_h2d(r.data(), host, (size_t)count * sizeof(float), reinterpret_cast<jst_stream_t>(g_stream)) != JST_OK)
        throw std::runtime_error(std::string("fromBuffer: ") + jst_last_error());
    return r;
}

Tensor Tensor::full(const Shape& shape, float value) {
    Tensor r(shape);
    core::fill(r.data(), value, r.size(), g_stream);
    check_cuda(cudaPeekAtLastError(), "fill");
    return r;
}

Tensor Tensor::randn(const Shape& shape) {
    Tensor r(shape);
    core::randn(r.data(), r.size(), g_randn_seed.fetch_add(1), g_stream);
    check_cuda(cudaPeekAtLastError(), "randn");
    return r;
}

std::vector<float> Tensor::to_array() const {
    std::vector<float> out((size_t)size());
    to_host(out.data());
    return out;
}

void Tensor::to_host(float* dst) const {
    if (size() == 0) return;
    const Tensor c = contiguous();  // strided views are gathered on the device first
    // waits for the core stream only
    if (jst_copy_d2h(dst, c.data(), (size_t)c.size() * sizeof(float), reinterpret_cast<jst_stream_t>(g_stream)) !=
        JST_OK)
        throw std::runtime_error(std::string("toArray: ") + jst_last_error());
}

Tensor Tensor::contiguous() const {
    if (is_contiguous()) return *this;
    if (ndim() > kMaxDims) throw std::runtime_error("contiguous: too many dims");
    Tensor r(shape_);
    StridedDesc d;
    d.ndim = ndim();
    for (int i = 0; i < d.ndim; ++i) {
        d.shape[i] = shape_[i];
        d.stride[i] = strides_[i];
    }
    strided_copy(data(), r.data(), d, size(), g_stream);
    check_cuda(cudaPeekAtLastError(), "strided copy");
    return r;
}

Tensor Tensor::transpose() const {
    if (ndim() != 2) throw std::runtime_error("transpose() requires 2D");
    return transpose(0, 1);
}

Tensor Tensor::transpose(int d0, int d1) const {
    d0 = norm_axis(d0, ndim());
    d1 = norm_axis(d1, ndim());
    Tensor r = *this;
    std::swap(r.shape_[d0], r.shape_[d1]);
    std::swap(r.strides_[d0], r.strides_[d1]);
    return r;
}

Tensor Tensor::view(const Shape& s) const {
    if (numel(s) != size()) throw std::runtime_error("View size mismatch");
    if (!is_contiguous()) throw std::runtime_error("View requires contiguous");
    Tensor r = *this;
    r.shape_ = s;
    r.strides_ = contiguous_strides(s);
    return r;
}

Tensor Tensor::reshape(const Shape& s) const {
    Shape res = s;
    int neg = -1;
    int64_t known = 1;
    for (int i = 0; i < (int)res.size(); ++i) {
        if (res[i] == -1) neg = i;
        else known *= res[i];
    }
    if (neg >= 0) res[neg] = known ? size() / known : 0;
    return is_contiguous() ? view(res) : contiguous().view(res);
}

// tensor.cpp:243-258: a view sharing the storage; negative bounds count from
// the end, `end` is clamped to the extent, and an empty range is an error.
Tensor Tensor::slice(int dim, int64_t start, int64_t end) const {
    dim = norm_axis(dim, ndim());
    if (start < 0) start += shape_[dim];
    if (end < 0) end += shape_[dim];
    if (end > shape_[dim]) end = shape_[dim];
    if (start < 0 || start >= end) throw std::runtime_error("slice: start >= end");
    Tensor r = *this;
    r.offset_ += start * strides_[dim];
    r.shape_[dim] = end - start;
    return r;
}

Tensor Tensor::squeeze(int axis) const {
    axis = norm_axis(axis, ndim());
    if (shape_[axis] != 1) throw std::runtime_error("Can only squeeze size-1");
    Tensor r = *this;
    r.shape_.erase(r.shape_.begin() + axis);
    r.strides_.erase(r.strides_.begin() + axis);
    return r;
}

Tensor Tensor::unsqueeze(int axis) const {
    axis = norm_axis(axis, ndim() + 1);
    Tensor r = *this;
    const int64_t st = axis < ndim() ? shape_[axis] * strides_[axis] : 1;
    r.shape_.insert(r.shape_.begin() + axis, 1);
    r.strides_.insert(r.strides_.begin() + axis, st);
    return r;
}

// Tensor::matmul -- reference native/core/tensor.cpp:630-654.
Tensor Tensor::matmul(const Tensor& other) const {
    if (ndim() == 2 && other.ndim() == 2) {
        const int64_t M = shape_[0], K = shape_[1], N = other.shape_[1];
        if (other.shape_[0] != K) throw std::runtime_error("matmul shape mismatch");
        Tensor r({M, N});
        gemm(*this, other, r, 1, nullptr);
        return r;
    }
    if (ndim() == 3 && other.ndim() == 3) {
        const int64_t B = shape_[0], M = shape_[1], K = shape_[2], N = other.shape_[2];
        if (other.shape_[0] != B || other.shape_[1] != K) throw std::runtime_error("matmul shape mismatch");
        Tensor r({B, M, N});
        gemm(*this, other, r, B, nullptr);
        return r;
    }
    if (ndim() == 2 && other.ndim() == 1) {  // matrix-vector: [M,K] x [K] -> [M]
        const int64_t M = shape_[0], K = shape_[1];
        if (other.shape_[0] != K) throw std::runtime_error("matmul shape mismatch");
        Tensor r({M, 1});
        gemm(*this, other.unsqueeze(1), r, 1, nullptr);
        return r.squeeze(1);
    }
    throw std::runtime_error("matmul: unsupported dims");
}

// Tensor::linear -- reference native/core/tensor.cpp:658-671: x [B,in] . w[out,in]^T + bias,
// one GEMM with the bias in its epilogue (the reference adds it in a second kernel).
Tensor Tensor::linear(const Tensor& weight, const Tensor* bias) const {
    if (ndim() != 2) throw std::runtime_error("linear: input must be 2D [B, in_f]");
    if (weight.ndim() != 2) throw std::runtime_error("linear: weight must be 2D [out_f, in_f]");
    const int64_t B = shape_[0], in_f = shape_[1], out_f = weight.shape_[0];
    if (weight.shape_[1] != in_f) throw std::runtime_error("linear: shape mismatch");
    if (bias && bias->size() != out_f) throw std::runtime_error("linear: bias size mismatch");
    Tensor r({B, out_f});
    gemm(*this, weight.transpose(), r, 1, bias);
    return r;
}

Tensor Tensor::add(const Tensor& other) const {
    if (shape_ == other.shape_) {
        const Tensor a = contiguous(), b = other.contiguous();
        Tensor r(shape_);
        core::add(a.data(), b.data(), r.data(), size(), g_stream);
        check_cuda(cudaPeekAtLastError(), "add");
        return r;
    }
    // [..., N] + [N] (or [1, N]): the bias broadcast of nn.Linear (nn.js:108)
    auto rowvec = [](const Tensor& big, const Tensor& v) {
        const int64_t n = big.shape().back();
        return big.ndim() >= 1 && v.size() == n && (v.ndim() == 1 || (v.ndim() == 2 && v.shape()[0] == 1));
    };
    const Tensor* big = nullptr;
    const Tensor* vec = nullptr;
    if (ndim() >= 2 && rowvec(*this, other)) { big = this; vec = &other; }
    else if (other.ndim() >= 2 && rowvec(other, *this)) { big = &other; vec = this; }
    if (!big) throw std::runtime_error("add: broadcast " + shape_str(shape_) + " + " + shape_str(other.shape_) +
                                       " not supported on this path");
    const Tensor a = big->contiguous(), v = vec->contiguous();
    Tensor r(big->shape());
    const int64_t cols = a.shape().back();
    core::add_rowvec(a.data(), v.data(), r.data(), a.size() / std::max<int64_t>(cols, 1), cols, g_stream);
    check_cuda(cudaPeekAtLastError(), "add");
    return r;
}

Tensor Tensor::relu() const {
    const Tensor a = contiguous();
    Tensor r(shape_);
    core::relu(a.data(), r.data(), size(), g_stream);
    check_cuda(cudaPeekAtLastError(), "relu");
    return r;
}

Tensor Tensor::relu_backward(const Tensor& x) const {
    if (x.shape_ != shape_) throw std::runtime_error("relu_backward: shape mismatch");
    const Tensor g = contiguous(), xc = x.contiguous();
    Tensor r(shape_);
    core::relu_backward(g.data(), xc.data(), r.data(), size(), g_stream);
    check_cuda(cudaPeekAtLastError(), "relu_backward");
    return r;
}

Tensor Tensor::sum(int dim, bool keepdim) const {
    dim = norm_axis(dim, ndim());
    const Tensor src = dim == 0 ? contiguous() : transpose(0, dim).contiguous();
    const int64_t rows = src.shape_[0];
    const int64_t cols = rows ? src.size() / rows : 0;
    Shape rest(src.shape_.begin() + 1, src.shape_.end());
    Tensor r(rest.empty() ? Shape{1} : rest);
    if (rows == 0) core::fill(r.data(), 0.0f, r.size(), g_stream);
    else core::sum_rows(src.data(), r.data(), rows, cols, g_stream);
    check_cuda(cudaPeekAtLastError(), "sum");
    // reduced layout is the transposed-order shape; restore the original order
    Shape out = shape_;
    out.erase(out.begin() + dim);
    if (dim != 0 && out.size() >= 1) {
        // src order after transpose(0, dim): [shape[dim], shape[1..dim-1], shape[0], shape[dim+1..]]
        Shape mid = rest;  // = [shape[1], ..., shape[dim-1], shape[0], shape[dim+1], ...]
        Tensor v = r.view(mid.empty() ? Shape{1} : mid);
        if (dim > 1) {
            // move shape[0] (now at position dim-1) back to the front by adjacent swaps
            for (int i = dim - 1; i > 0; --i) v = v.transpose(i, i - 1);
        }
        r = v.contiguous();
    }
    if (keepdim) {
        Shape k = shape_;
        k[dim] = 1;
        return r.reshape(k);
    }
    return out.empty() ? r.reshape({1}) : r.reshape(out);
}

}  // namespace core
}  // namespace jst
