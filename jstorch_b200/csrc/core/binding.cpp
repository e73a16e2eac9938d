// binding.cpp -- Python module `jstorch_b200._core`: the host core's Tensor and
// GradTensor with the method names of the reference's N-API binding
// (native/binding/napi.cpp: TensorWrap :61-759, GradTensorWrap :762-1485), so
// tests drive the same calls a JsTorch program makes (Node is not available
// to run the JS surface itself).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "autograd.h"
#include "compiled.h"
#include "../../../include/jstorch_gemm.h"
#include "core_kernels.h"

namespace py = pybind11;
using jst::core::GradPtr;
using jst::core::GradTensor;
using jst::core::Shape;
using jst::core::Tensor;

namespace {

Shape to_shape(const py::object& o) {
    Shape s;
    for (auto h : o) s.push_back(h.cast<int64_t>());
    return s;
}

// Tensor.fromBuffer(Float32Array, shape) -- napi.cpp:702-707
Tensor from_buffer(py::array_t<float, py::array::c_style | py::array::forcecast> a, const py::object& shape) {
    Shape s = shape.is_none() ? Shape(a.shape(), a.shape() + a.ndim()) : to_shape(shape);
    return Tensor::from_buffer(a.data(), (int64_t)a.size(), s);
}

// toArray -- napi.cpp:235-238 returns nested JS arrays; here a numpy array of
// the tensor's shape, filled in place from the pinned staging
py::array_t<float> to_array(const Tensor& t) {
    std::vector<py::ssize_t> shp(t.shape().begin(), t.shape().end());
    py::array_t<float> out(shp);
    t.to_host(out.mutable_data());
    return out;
}

// toFloat32Array -- the flat Float32Array form (no nested arrays, napi.cpp:17-30)
py::array_t<float> to_float32_array(const Tensor& t) {
    py::array_t<float> out((py::ssize_t)t.size());
    t.to_host(out.mutable_data());
    return out;
}

GradPtr as_grad(const py::object& o) {
    if (py::isinstance<GradTensor>(o)) return o.cast<GradPtr>();
    if (py::isinstance<Tensor>(o)) return GradTensor::make(o.cast<Tensor>(), false);
    throw py::type_error("expected a Tensor or GradTensor");
}

}  // namespace

PYBIND11_MODULE(_core, m) {
    m.doc() = "host core of the jstorch_b200 matmul path (Tensor, GradTensor)";
    py::register_exception<std::runtime_error>(m, "JsTorchError", PyExc_RuntimeError);

    py::class_<Tensor>(m, "Tensor")
        .def_static("fromBuffer", &from_buffer, py::arg("data"), py::arg("shape") = py::none())
        .def_static("zeros", [](const py::object& s) { return Tensor::zeros(to_shape(s)); })
        .def_static("full", [](const py::object& s, float v) { return Tensor::full(to_shape(s), v); })
        .def_static("randn", [](const py::object& s) { return Tensor::randn(to_shape(s)); })
        .def_property_readonly("shape", [](const Tensor& t) { return std::vector<int64_t>(t.shape()); })
        .def_property_readonly("strides", [](const Tensor& t) { return std::vector<int64_t>(t.strides()); })
        .def("size", &Tensor::size)
        .def("isContiguous", &Tensor::is_contiguous)
        .def("contiguous", &Tensor::contiguous)
        .def("toArray", &to_array)
        .def("toFloat32Array", &to_float32_array)
        .def("data_ptr", [](const Tensor& t) { return reinterpret_cast<uintptr_t>(t.data()); })
        .def("matmul", &Tensor::matmul)
        .def("linear", [](const Tensor& x, const Tensor& w, const py::object& b) {
                if (b.is_none()) return x.linear(w, nullptr);
                Tensor bt = b.cast<Tensor>();
                return x.linear(w, &bt);
            }, py::arg("weight"), py::arg("bias") = py::none())
        .def("add", &Tensor::add)
        .def("relu", &Tensor::relu)
        .def("sum", &Tensor::sum, py::arg("dim"), py::arg("keepdim") = false)
        .def("transpose", [](const Tensor& t, py::args dims) {
                if (dims.size() == 0) return t.transpose();
                if (dims.size() == 2) return t.transpose(dims[0].cast<int>(), dims[1].cast<int>());
                throw py::type_error("transpose() takes no or two dims");
            })
        .def("reshape", [](const Tensor& t, const py::object& s) { return t.reshape(to_shape(s)); })
        .def("unsqueeze", &Tensor::unsqueeze)
        .def("squeeze", &Tensor::squeeze)
        .def("slice", &Tensor::slice, "slice(dim, start, end): a view (napi slice, tensor.cpp:243-258)");

    py::class_<GradTensor, GradPtr>(m, "GradTensor")
        .def(py::init([](const Tensor& t, bool rg) { return GradTensor::make(t, rg); }), py::arg("tensor"),
             py::arg("requires_grad") = false)
        .def_property_readonly("data", [](const GradTensor& g) { return g.data; })
        .def_property("requires_grad", [](const GradTensor& g) { return g.requires_grad; },
                      [](GradTensor& g, bool v) { g.requires_grad = v; })
        .def_property_readonly("grad", [](const GradTensor& g) -> py::object {
                if (!g.has_grad || !g.grad_) return py::none();
                return py::cast(*g.grad_);
            })
        .def_property_readonly("shape", [](const GradTensor& g) { return std::vector<int64_t>(g.data.shape()); })
        .def("toArray", [](const GradTensor& g) { return to_array(g.data); })
        .def("matmul", [](GradTensor& self, const py::object& o) { return self.shared_from_this()->matmul_(as_grad(o)); })
        .def("add", [](GradTensor& self, const py::object& o) { return self.shared_from_this()->add_(as_grad(o)); })
        .def("relu", [](GradTensor& self) { return self.shared_from_this()->relu_(); })
        .def("transpose", [](GradTensor& self, py::args dims) {
                if (dims.size() == 0) return self.shared_from_this()->transpose_();
                if (dims.size() == 2) return self.shared_from_this()->transpose_(dims[0].cast<int>(), dims[1].cast<int>());
                throw py::type_error("transpose() takes no or two dims");
            })
        // backward(upstream = ones(shape)) -- napi.cpp:974-980
        .def("backward", [](GradTensor& self, const py::object& up) {
                Tensor u = up.is_none() ? Tensor::full(self.data.shape(), 1.0f) : up.cast<Tensor>();
                GradTensor::backward(self.shared_from_this(), u);
            }, py::arg("upstream") = py::none())
        .def("zero_grad", [](GradTensor& g) { g.grad_.reset(); g.has_grad = false; });

    // CompiledGraph -- napi.cpp:1488-1830 (slot builders :1562-1574, run :1785).  run() here
    // takes (input, params) and returns (output, [grad per param]); the reference's
    // target / Adam arguments belong to its optimizer, which is not on this path.
    py::class_<jst::core::CompiledGraph>(m, "CompiledGraph")
        .def(py::init<>())
        .def("input", &jst::core::CompiledGraph::input)
        .def("param", &jst::core::CompiledGraph::param)
        .def("matmul", &jst::core::CompiledGraph::matmul)
        .def("transpose", &jst::core::CompiledGraph::transpose)
        .def("add", &jst::core::CompiledGraph::add)
        .def("relu", &jst::core::CompiledGraph::relu)
        .def("setOutput", &jst::core::CompiledGraph::set_output)
        .def("run", [](jst::core::CompiledGraph& g, const Tensor& x, const std::vector<Tensor>& params) {
                std::vector<Tensor> grads;
                Tensor y = g.run(x, params, grads);
                return py::make_tuple(y, grads);
            })
        .def_property_readonly("fused", &jst::core::CompiledGraph::fused)
        .def_property_readonly("replaying", &jst::core::CompiledGraph::replaying)
        .def_property_readonly("kernelsPerRun", &jst::core::CompiledGraph::kernels_per_run);

    m.def("clearCache", &jst::core::clear_cache, "synchronise and drop cached device blocks (napi.cpp:755)");
    m.def("reservedBytes", &jst::core::reserved_bytes);
    m.def("stridedCopies", &jst::core::strided_copy_count,
          "number of contiguous() materialisations (strided copies) so far");
    m.def("cachedBytes", &jst::core::cached_bytes);
    m.def("releaseHostStaging", [] { jst_release_caches(); },
          "free the pinned fromBuffer / toArray staging (and the GEMM library's other caches)");
}
