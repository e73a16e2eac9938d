// autograd.cpp -- GradTensor ops and backward engine (see autograd.h).
#include "autograd.h"

#include <stdexcept>

namespace jst {
namespace core {

GradPtr GradTensor::make_with_grad(Tensor out, GradFn fn, std::vector<GradPtr> ps) {
    auto r = std::make_shared<GradTensor>(std::move(out), true);
    r->grad_fn = std::move(fn);
    r->parents = std::move(ps);
    return r;
}

void GradTensor::topo_sort(GradTensor* node, std::vector<GradTensor*>& order,
                           std::unordered_set<GradTensor*>& seen) {
    if (!node || seen.count(node) || !node->requires_grad) return;
    seen.insert(node);
    for (auto& p : node->parents)
        if (p) topo_sort(p.get(), order, seen);
    order.push_back(node);
}

void GradTensor::backward(const GradPtr& root, Tensor upstream) {
    if (upstream.shape() != root->data.shape())
        throw std::runtime_error("backward: upstream shape " + shape_str(upstream.shape()) + " != output shape " +
                                 shape_str(root->data.shape()));
    std::vector<GradTensor*> order;
    std::unordered_set<GradTensor*> seen;
    topo_sort(root.get(), order, seen);
    root->grad_ = std::make_shared<Tensor>(std::move(upstream));
    root->has_grad = true;
    for (int i = (int)order.size() - 1; i >= 0; --i) {
        GradTensor* node = order[i];
        if (!node->grad_fn || !node->has_grad) continue;
        std::vector<bool> needed(node->parents.size());
        for (size_t j = 0; j < node->parents.size(); ++j)
            needed[j] = node->parents[j] && node->parents[j]->requires_grad;
        auto grads = node->grad_fn(*node->grad_, needed);
        for (size_t j = 0; j < node->parents.size(); ++j) {
            auto& p = node->parents[j];
            if (!needed[j] || j >= grads.size() || !grads[j].defined()) continue;
            if (p->has_grad) {
                *p->grad_ = p->grad_->add(grads[j]);
            } else {
                p->grad_ = std::make_shared<Tensor>(std::move(grads[j]));
                p->has_grad = true;
            }
        }
    }
}

// forward a.b; backward {g.b^T, a^T.g} (autograd.hpp:433-441).  The transposes
// are views: the GEMMs run as NT and TN with no copies.
GradPtr GradTensor::matmul_(const GradPtr& other) {
    Tensor out = data.matmul(other->data);
    if (!requires_grad && !other->requires_grad) return make(std::move(out));
    Tensor a = data, b = other->data;
    return make_with_grad(
        std::move(out),
        [a, b](const Tensor& g, const std::vector<bool>& need) {
            std::vector<Tensor> r(2);
            if (a.ndim() == 2 && b.ndim() == 2) {
                if (need[0]) r[0] = g.matmul(b.transpose());
                if (need[1]) r[1] = a.transpose().matmul(g);
            } else if (a.ndim() == 3 && b.ndim() == 3) {
                if (need[0]) r[0] = g.matmul(b.transpose(1, 2));
                if (need[1]) r[1] = a.transpose(1, 2).matmul(g);
            } else {
                throw std::runtime_error("matmul backward: unsupported dims");
            }
            return r;
        },
        {shared_from_this(), other});
}

// autograd.hpp:324-332: sum away leading dims, then keep-dim sums over size-1 dims.
Tensor GradTensor::unbroadcast(const Tensor& grad, const Shape& target) {
    Tensor g = grad;
    while (g.ndim() > (int)target.size()) g = g.sum(0, false);
    for (int i = 0; i < (int)target.size(); ++i)
        if (target[i] == 1 && g.shape()[i] != 1) g = g.sum(i, true);
    return g;
}

GradPtr GradTensor::add_(const GradPtr& other) {
    Tensor out = data.add(other->data);
    if (!requires_grad && !other->requires_grad) return make(std::move(out));
    const Shape sa = data.shape(), sb = other->data.shape();
    return make_with_grad(
        std::move(out),
        [sa, sb](const Tensor& g, const std::vector<bool>& need) {
            std::vector<Tensor> r(2);
            if (need[0]) r[0] = unbroadcast(g, sa);
            if (need[1]) r[1] = unbroadcast(g, sb);
            return r;
        },
        {shared_from_this(), other});
}

// relu'(x) = 1 where x > 0, else 0 (0 at x == 0), autograd.hpp:127-134.
GradPtr GradTensor::relu_() {
    Tensor out = data.relu();
    if (!requires_grad) return make(std::move(out));
    Tensor x = data;
    return make_with_grad(
        std::move(out),
        [x](const Tensor& g, const std::vector<bool>&) { return std::vector<Tensor>{g.relu_backward(x)}; },
        {shared_from_this()});
}

GradPtr GradTensor::transpose_() {
    Tensor out = data.transpose();
    if (!requires_grad) return make(std::move(out));
    return make_with_grad(
        std::move(out), [](const Tensor& g, const std::vector<bool>&) { return std::vector<Tensor>{g.transpose()}; },
        {shared_from_this()});
}

GradPtr GradTensor::transpose_(int d0, int d1) {
    Tensor out = data.transpose(d0, d1);
    if (!requires_grad) return make(std::move(out));
    return make_with_grad(
        std::move(out),
        [d0, d1](const Tensor& g, const std::vector<bool>&) { return std::vector<Tensor>{g.transpose(d0, d1)}; },
        {shared_from_this()});
}

}  // namespace core
}  // namespace jst
