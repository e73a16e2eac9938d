// autograd.h -- reverse-mode autograd of the host core for the matmul path:
// the reference's GradTensor (native/core/autograd.hpp:18-851) restricted to
// the ops nn.Linear / ReLU / Sequential reach (matmul_, add_, relu_,
// transpose_) and the backward engine.
//
// Differences from the reference:
//   * a grad function receives which parents need a gradient, so matmul_
//     skips the GEMM of a parent that does not (the reference computes both
//     g.b^T and a^T.g and discards one, autograd.hpp:439 and :55);
//   * the transposed operands of those GEMMs are views consumed by the NT / TN
//     kernels (no contiguous copies);
//   * relu_'s gradient is one fused kernel instead of full + gt + mul (:132).
#pragma once
#include <functional>
#include <memory>
#include <unordered_set>
#include <vector>

#include "tensor.h"

namespace jst {
namespace core {

class GradTensor;
using GradPtr = std::shared_ptr<GradTensor>;

class GradTensor : public std::enable_shared_from_this<GradTensor> {
  public:
    // grads[i] for parent i; entries for parents with needed[i] == false may be empty
    using GradFn = std::function<std::vector<Tensor>(const Tensor& g, const std::vector<bool>& needed)>;

    Tensor data;
    bool requires_grad = false;
    std::shared_ptr<Tensor> grad_;
    bool has_grad = false;
    GradFn grad_fn;
    std::vector<GradPtr> parents;

    explicit GradTensor(Tensor d, bool rg = false) : data(std::move(d)), requires_grad(rg) {}

    static GradPtr make(Tensor d, bool rg = false) { return std::make_shared<GradTensor>(std::move(d), rg); }

    // autograd.hpp:40-65: topological sort from the root, reverse sweep,
    // gradients accumulated with Tensor::add.
    static void backward(const GradPtr& root, Tensor upstream);

    GradPtr matmul_(const GradPtr& other);   // autograd.hpp:433-441
    GradPtr add_(const GradPtr& other);      // autograd.hpp:334-342 (+ unbroadcast :324-332)
    GradPtr relu_();                         // autograd.hpp:127-134
    GradPtr transpose_();                    // autograd.hpp:532-538
    GradPtr transpose_(int d0, int d1);      // autograd.hpp:524-530

    static Tensor unbroadcast(const Tensor& grad, const Shape& target);

  private:
    GradPtr make_with_grad(Tensor out, GradFn fn, std::vector<GradPtr> ps);
    static void topo_sort(GradTensor* node, std::vector<GradTensor*>& order, std::unordered_set<GradTensor*>& seen);
};

}  // namespace core
}  // namespace jst
