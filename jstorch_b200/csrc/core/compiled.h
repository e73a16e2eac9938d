// compiled.h -- CompiledGraph of the host core: a recorded tape of matmul-path
// ops replayed as one forward + backward (reference: CompiledGraph,
// native/core/autograd.hpp:856-1498, built through CompiledGraphWrap,
// native/binding/napi.cpp:1488-1830; its MATMUL case :1134, backward + Adam
// :1486-1495).
//
// B200 form of the same idea:
//   * the tape is pattern-matched into Linear layers: matmul(x, transpose(W))
//     -> add(b) -> [relu] becomes ONE GEMM with the bias and ReLU in its
//     epilogue;
//   * backward per layer: dW = g^T . x (TN GEMM, straight into [out, in]),
//     db = column sum of g, and the input gradient g . W (NN GEMM) with the
//     previous layer's ReLU mask fused into its epilogue;
//   * the weight / bias gradients of a layer run on a second stream, forked
//     once the layer's upstream gradient exists and joined at the end, so the
//     graph has two branches: the input-gradient chain and the parameter
//     gradients that hang off it;
//   * the first run executes eagerly (allocating every buffer), the second
//     captures the whole pass into a CUDA graph, later runs replay it with one
//     launch.  Buffers (activations, gradients) belong to the graph object.
// Tapes that are not a chain of Linear(+ReLU) layers run eagerly through
// GradTensor.  The optimizer step of the reference's run() is not part of
// this path.
#pragma once
#include <cuda_runtime.h>

#include <memory>
#include <vector>

#include "tensor.h"

namespace jst {
namespace core {

class CompiledGraph {
  public:
    CompiledGraph();
    ~CompiledGraph();
    CompiledGraph(const CompiledGraph&) = delete;
    CompiledGraph& operator=(const CompiledGraph&) = delete;

    // tape builders: each returns the slot of its result
    int input();
    int param();
    int matmul(int a, int b);
    int transpose(int a);
    int add(int a, int b);
    int relu(int a);
    void set_output(int slot);

    // One forward + backward with loss = sum(output) (upstream = ones, as
    // GradTensor::backward's default).  `params` are in param() order and must
    // be the same device tensors on every call once the graph is captured (a
    // different set re-captures).  Returns the output; grads receives one
    // contiguous gradient per parameter.  The returned tensors are the graph's
    // own buffers and are overwritten by the next run.
    Tensor run(const Tensor& input, const std::vector<Tensor>& params, std::vector<Tensor>& grads);

    bool fused() const { return fused_; }    // the tape was recognised as Linear layers
    bool replaying() const { return exec_ != nullptr; }
    int kernels_per_run() const { return kernels_per_run_; }  // kernel nodes of the captured graph

  private:
    struct Op {
        enum Kind { INPUT, PARAM, MATMUL, TRANSPOSE, ADD, RELU } kind;
        int a = -1, b = -1;
        int param_index = -1;
    };
    struct Layer {
        int w = -1, b = -1;  // param indices (b = -1: no bias)
        bool relu = false;
        int64_t in = 0, out = 0;
    };

    bool plan();  // recognise the Linear chain; false -> eager fallback
    void alloc_buffers(int64_t batch);
    void enqueue(cudaStream_t s, const std::vector<Tensor>& params);
    Tensor run_eager(const Tensor& input, const std::vector<Tensor>& params, std::vector<Tensor>& grads);

    std::vector<Op> ops_;
    int input_slot_ = -1, out_slot_ = -1, n_params_ = 0;
    bool planned_ = false, fused_ = false;
    std::vector<Layer> layers_;

    // buffers of the fused plan
    int64_t batch_ = -1;
    Tensor x_;                  // copy of the input
    std::vector<Tensor> act_;   // layer outputs (post-ReLU where present)
    std::vector<Tensor> g_;     // gradient w.r.t. each layer's pre-activation
    std::vector<Tensor> grads_; // parameter gradients
    Tensor ones_;

    cudaStream_t stream_ = nullptr, side_ = nullptr;
    cudaEvent_t ev_in_ = nullptr, ev_out_ = nullptr, ev_side_ = nullptr;
    std::vector<cudaEvent_t> ev_g_;  // per layer: its upstream gradient is ready
    cudaGraphExec_t exec_ = nullptr;
    std::vector<const float*> captured_params_;
    int runs_ = 0;
    int kernels_per_run_ = 0;
};

}  // namespace core
}  // namespace jst
