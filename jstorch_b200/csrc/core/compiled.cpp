// compiled.cpp -- CompiledGraph (see compiled.h).
#include "compiled.h"

#include <stdexcept>
#include <string>

#include "../../../include/jstorch_gemm.h"
#include "autograd.h"
#include "core_kernels.h"

namespace jst {
namespace core {

namespace {
void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) {
        cudaGetLastError();
        throw std::runtime_error(std::string("CompiledGraph: ") + what + ": " + cudaGetErrorString(e));
    }
}

void ckj(int rc, const char* what) {
    if (rc != JST_OK) throw std::runtime_error(std::string("CompiledGraph: ") + what + ": " + jst_last_error());
}

// row-major GEMM on stream s: C[M,N] = op(A) op(B) with the given epilogue
void gemm(cudaStream_t s, int transA, int transB, int M, int N, int K, const float* A, int64_t lda, const float* B,
          int64_t ldb, float* C, const float* bias, int epilogue, const float* aux) {
    jst_gemm_desc d;
    jst_gemm_desc_init(&d, M, N, K, A, B, C);
    d.transA = transA;
    d.transB = transB;
    d.lda = lda;
    d.ldb = ldb;
    d.bias = bias;
    d.epilogue = epilogue;
    d.aux = aux;
    d.ld_aux = N;
    d.stream = reinterpret_cast<jst_stream_t>(s);
    ckj(jst_gemm_ex(&d), "GEMM");
}
}  // namespace

CompiledGraph::CompiledGraph() {
    ck(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream create");
    ck(cudaStreamCreateWithFlags(&side_, cudaStreamNonBlocking), "stream create");
    ck(cudaEventCreateWithFlags(&ev_in_, cudaEventDisableTiming), "event create");
    ck(cudaEventCreateWithFlags(&ev_out_, cudaEventDisableTiming), "event create");
    ck(cudaEventCreateWithFlags(&ev_side_, cudaEventDisableTiming), "event create");
}

CompiledGraph::~CompiledGraph() {
    if (stream_) cudaStreamSynchronize(stream_);
    if (exec_) cudaGraphExecDestroy(exec_);
    if (side_) cudaStreamSynchronize(side_);
    if (ev_in_) cudaEventDestroy(ev_in_);
    if (ev_out_) cudaEventDestroy(ev_out_);
    if (ev_side_) cudaEventDestroy(ev_side_);
    for (auto e : ev_g_) cudaEventDestroy(e);
    if (side_) cudaStreamDestroy(side_);
    if (stream_) cudaStreamDestroy(stream_);
}

int CompiledGraph::input() {
    if (input_slot_ >= 0) throw std::runtime_error("CompiledGraph: one input only");
    ops_.push_back({Op::INPUT});
    input_slot_ = (int)ops_.size() - 1;
    return input_slot_;
}

int CompiledGraph::param() {
    Op o{Op::PARAM};
    o.param_index = n_params_++;
    ops_.push_back(o);
    return (int)ops_.size() - 1;
}

static void check_slot(int s, size_t n) {
    if (s < 0 || (size_t)s >= n) throw std::runtime_error("CompiledGraph: bad slot");
}

int CompiledGraph::matmul(int a, int b) {
    check_slot(a, ops_.size());
    check_slot(b, ops_.size());
    ops_.push_back({Op::MATMUL, a, b});
    return (int)ops_.size() - 1;
}

int CompiledGraph::transpose(int a) {
    check_slot(a, ops_.size());
    ops_.push_back({Op::TRANSPOSE, a});
    return (int)ops_.size() - 1;
}

int CompiledGraph::add(int a, int b) {
    check_slot(a, ops_.size());
    check_slot(b, ops_.size());
    ops_.push_back({Op::ADD, a, b});
    return (int)ops_.size() - 1;
}

int CompiledGraph::relu(int a) {
    check_slot(a, ops_.size());
    ops_.push_back({Op::RELU, a});
    return (int)ops_.size() - 1;
}

void CompiledGraph::set_output(int slot) {
    check_slot(slot, ops_.size());
    out_slot_ = slot;
    planned_ = false;
}

// Walk back from the output: [relu] <- add(bias param) <- matmul(x, transpose(W param)),
// x being the previous layer's output or the input; every intermediate slot used once.
bool CompiledGraph::plan() {
    layers_.clear();
    if (input_slot_ < 0 || out_slot_ < 0) return false;
    std::vector<int> uses(ops_.size(), 0);
    for (auto& o : ops_) {
        if (o.a >= 0) ++uses[o.a];
        if (o.b >= 0) ++uses[o.b];
    }
    auto is_param = [&](int s) { return s >= 0 && ops_[s].kind == Op::PARAM; };
    std::vector<Layer> rev;
    int cur = out_slot_;
    while (cur != input_slot_) {
        Layer L;
        if (ops_[cur].kind == Op::RELU) {
            L.relu = true;
            cur = ops_[cur].a;
            if (uses[cur] != 1) return false;
        }
        if (ops_[cur].kind == Op::ADD) {
            const int x = ops_[cur].a, y = ops_[cur].b;
            const int mm = is_param(y) ? x : (is_param(x) ? y : -1);
            if (mm < 0 || uses[mm] != 1) return false;
            L.b = ops_[is_param(y) ? y : x].param_index;
            cur = mm;
        }
        if (ops_[cur].kind != Op::MATMUL) return false;
        const int t = ops_[cur].b;
        if (ops_[t].kind != Op::TRANSPOSE || uses[t] != 1 || !is_param(ops_[t].a)) return false;
        L.w = ops_[ops_[t].a].param_index;
        rev.push_back(L);
        cur = ops_[cur].a;
        if (cur != input_slot_ && uses[cur] != 1) return false;
        if (cur != input_slot_ && ops_[cur].kind == Op::PARAM) return false;
    }
    if (rev.empty()) return false;
    layers_.assign(rev.rbegin(), rev.rend());
    return true;
}

void CompiledGraph::alloc_buffers(int64_t batch) {
    batch_ = batch;
    x_ = Tensor({batch, layers_.front().in});
    act_.clear();
    g_.clear();
    for (auto& L : layers_) {
        act_.emplace_back(Shape{batch, L.out});
        g_.emplace_back(Shape{batch, L.out});
    }
    ones_ = Tensor::full({batch, layers_.back().out}, 1.0f);
    while (ev_g_.size() < layers_.size()) {
        cudaEvent_t e = nullptr;
        ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event create");
        ev_g_.push_back(e);
    }
}

// forward + backward of the Linear chain on stream s (no host synchronisation,
// so it can be captured into a CUDA graph)
void CompiledGraph::enqueue(cudaStream_t s, const std::vector<Tensor>& params) {
    const int L = (int)layers_.size();
    const int64_t B = batch_;
    for (int l = 0; l < L; ++l) {  // y = relu?(x . W^T + b): NT GEMM, bias / ReLU in the epilogue
        const Layer& ly = layers_[l];
        const Tensor& x = l == 0 ? x_ : act_[l - 1];
        const float* bias = ly.b >= 0 ? params[ly.b].data() : nullptr;
        const int epi = (bias ? JST_EPI_BIAS : 0) | (ly.relu ? JST_EPI_RELU : 0);
        gemm(s, 0, 1, (int)B, (int)ly.out, (int)ly.in, x.data(), ly.in, params[ly.w].data(), ly.in, act_[l].data(),
             bias, epi, nullptr);
    }
    // gradient w.r.t. the last pre-activation: the ones seed, masked when the last layer has a ReLU
    const Layer& last = layers_.back();
    if (last.relu) core::relu_backward(ones_.data(), act_[L - 1].data(), g_[L - 1].data(), B * last.out, s);
    for (int l = L - 1; l >= 0; --l) {
        const Layer& ly = layers_[l];
        const Tensor& x = l == 0 ? x_ : act_[l - 1];
        const float* g = (l == L - 1 && !last.relu) ? ones_.data() : g_[l].data();
        // parameter gradients on the side stream, once g exists
        ck(cudaEventRecord(ev_g_[l], s), "event record");
        ck(cudaStreamWaitEvent(side_, ev_g_[l], 0), "stream wait");
        // dW [out, in] = g^T . x   (TN)
        gemm(side_, 1, 0, (int)ly.out, (int)ly.in, (int)B, g, ly.out, x.data(), ly.in, grads_[ly.w].data(), nullptr,
             JST_EPI_NONE, nullptr);
        if (ly.b >= 0) core::sum_rows(g, grads_[ly.b].data(), B, ly.out, side_);
        // gradient of the previous layer's pre-activation: (g . W) masked by its ReLU (NN)
        if (l > 0) {
            const bool mask = layers_[l - 1].relu;
            gemm(s, 0, 0, (int)B, (int)ly.in, (int)ly.out, g, ly.out, params[ly.w].data(), ly.in, g_[l - 1].data(),
                 nullptr, mask ? JST_EPI_MASK : JST_EPI_NONE, mask ? act_[l - 1].data() : nullptr);
        }
    }
    ck(cudaEventRecord(ev_side_, side_), "event record");  // join
    ck(cudaStreamWaitEvent(s, ev_side_, 0), "stream wait");
    ck(cudaPeekAtLastError(), "launch");
}

Tensor CompiledGraph::run_eager(const Tensor& input, const std::vector<Tensor>& params, std::vector<Tensor>& grads) {
    std::vector<GradPtr> slots(ops_.size());
    std::vector<GradPtr> ps;
    for (size_t i = 0; i < ops_.size(); ++i) {
        const Op& o = ops_[i];
        switch (o.kind) {
            case Op::INPUT: slots[i] = GradTensor::make(input, false); break;
            case Op::PARAM:
                slots[i] = GradTensor::make(params[o.param_index], true);
                ps.push_back(slots[i]);
                break;
            case Op::MATMUL: slots[i] = slots[o.a]->matmul_(slots[o.b]); break;
            case Op::TRANSPOSE: slots[i] = slots[o.a]->transpose_(); break;
            case Op::ADD: slots[i] = slots[o.a]->add_(slots[o.b]); break;
            case Op::RELU: slots[i] = slots[o.a]->relu_(); break;
        }
    }
    GradPtr y = slots[out_slot_];
    GradTensor::backward(y, Tensor::full(y->data.shape(), 1.0f));
    grads.clear();
    for (auto& p : ps) grads.push_back(p->has_grad ? p->grad_->contiguous() : Tensor::zeros(p->data.shape()));
    return y->data;
}

Tensor CompiledGraph::run(const Tensor& input, const std::vector<Tensor>& params, std::vector<Tensor>& grads) {
    if (out_slot_ < 0) throw std::runtime_error("CompiledGraph: setOutput() not called");
    if ((int)params.size() != n_params_) throw std::runtime_error("CompiledGraph: wrong number of parameters");
    if (!planned_) {
        fused_ = plan();
        planned_ = true;
        if (fused_) {
            for (auto& ly : layers_) {  // shapes from the weights [out, in]
                const Tensor& w = params[ly.w];
                if (w.ndim() != 2) throw std::runtime_error("CompiledGraph: weights must be 2-D");
                ly.out = w.shape()[0];
                ly.in = w.shape()[1];
                if (ly.b >= 0 && params[ly.b].size() != ly.out)
                    throw std::runtime_error("CompiledGraph: bias size mismatch");
            }
            for (size_t l = 1; l < layers_.size(); ++l)
                if (layers_[l].in != layers_[l - 1].out) throw std::runtime_error("CompiledGraph: layer shape mismatch");
            grads_.clear();  // zero: a parameter outside the chain keeps a zero gradient
            for (auto& p : params) grads_.push_back(Tensor::zeros(p.shape()));
        }
    }
    if (!fused_) return run_eager(input, params, grads);

    if (input.ndim() != 2 || input.shape()[1] != layers_.front().in)
        throw std::runtime_error("CompiledGraph: input must be [batch, " + std::to_string(layers_.front().in) + "]");
    for (size_t i = 0; i < params.size(); ++i)
        if (!params[i].is_contiguous() || params[i].shape() != grads_[i].shape())
            throw std::runtime_error("CompiledGraph: parameter " + std::to_string(i) +
                                     " must be contiguous with the shape of the first run");
    if (input.shape()[0] != batch_) {  // (re)size the buffers; a new graph is captured
        alloc_buffers(input.shape()[0]);
        if (exec_) cudaGraphExecDestroy(exec_);
        exec_ = nullptr;
        runs_ = 0;
    }
    std::vector<const float*> addrs;
    for (auto& p : params) addrs.push_back(p.data());
    if (exec_ && addrs != captured_params_) {  // other parameter tensors: capture again
        cudaGraphExecDestroy(exec_);
        exec_ = nullptr;
        runs_ = 1;
    }

    const Tensor in = input.contiguous();
    // ordered after earlier core work (legacy stream) and back again at the end
    ck(cudaEventRecord(ev_in_, core_stream()), "event record");
    ck(cudaStreamWaitEvent(stream_, ev_in_, 0), "stream wait");
    ck(cudaMemcpyAsync(x_.data(), in.data(), (size_t)in.size() * 4, cudaMemcpyDeviceToDevice, stream_), "input copy");
    if (runs_ == 0) {
        enqueue(stream_, params);  // first run: eager, initialises every library resource
    } else {
        if (!exec_) {
            cudaGraph_t g = nullptr;
            ck(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
            try {
                enqueue(stream_, params);
            } catch (...) {
                cudaStreamEndCapture(stream_, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            ck(cudaStreamEndCapture(stream_, &g), "end capture");
            size_t n = 0;
            cudaGraphGetNodes(g, nullptr, &n);
            std::vector<cudaGraphNode_t> nodes(n);
            if (n) cudaGraphGetNodes(g, nodes.data(), &n);
            kernels_per_run_ = 0;
            for (auto nd : nodes) {
                cudaGraphNodeType t;
                if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels_per_run_;
            }
            const cudaError_t e = cudaGraphInstantiate(&exec_, g, 0);
            cudaGraphDestroy(g);
            ck(e, "graph instantiate");
            captured_params_ = addrs;
        }
        ck(cudaGraphLaunch(exec_, stream_), "graph launch");
    }
    ck(cudaEventRecord(ev_out_, stream_), "event record");
    ck(cudaStreamWaitEvent(core_stream(), ev_out_, 0), "stream wait");
    ++runs_;
    grads = grads_;
    return act_.back();
}

}  // namespace core
}  // namespace jst
