"""Python mirror of the part of the reference's src/nn.js that feeds the
matmul path: Module (nn.js:7-93), Linear (:96-111), ReLU (:547) and
Sequential (:560-569), over the host core's Tensor / GradTensor.

In JsTorch these classes stay JavaScript and are unchanged by the drop-in;
Node is not available here, so this mirror reproduces their exact
composition (x.matmul(W.transpose()).add(b), parameters wrapped by
_init_grad, load_state_dict replacing parameters) for the tests and the
benchmark.  All arithmetic runs in the native core.
"""
from __future__ import annotations

from ._core import GradTensor, Tensor


class Module:
    """nn.js:7-93."""

    def __init__(self):
        self._parameters: dict = {}
        self._modules: dict = {}
        self.training = True

    def parameters(self) -> list:
        out = [p for p in self._parameters.values() if p is not None]
        for m in self._modules.values():
            out.extend(m.parameters())
        return out

    def _init_grad(self) -> "Module":
        """nn.js:28-40: wrap every parameter as GradTensor(requires_grad=True)."""
        for name, p in list(self._parameters.items()):
            if p is None:
                continue
            if isinstance(p, GradTensor):
                p.requires_grad = True
            else:
                self._parameters[name] = GradTensor(p, True)
        for m in self._modules.values():
            m._init_grad()
        return self

    def load_state_dict(self, state: dict, prefix: str = "") -> None:
        """nn.js:58-80: replace parameters by key (call _init_grad afterwards)."""
        for name in list(self._parameters):
            key = f"{prefix}.{name}" if prefix else name
            if key in state:
                self._parameters[name] = state[key]
        for name, m in self._modules.items():
            m.load_state_dict(state, f"{prefix}.{name}" if prefix else name)

    def forward(self, *args):
        raise NotImplementedError("forward() must be implemented")

    def __call__(self, *args):
        return self.forward(*args)


class Linear(Module):
    """nn.js:96-111: weight [out, in] ~ Tensor.randn, bias zeros [out]."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self._parameters["weight"] = Tensor.randn([out_features, in_features])
        self._parameters["bias"] = Tensor.zeros([out_features]) if bias else None

    def forward(self, x):
        # nn.js:105-110: x.matmul(W.transpose()) then .add(bias)
        out = x.matmul(self._parameters["weight"].transpose())
        if self._parameters.get("bias") is not None:
            out = out.add(self._parameters["bias"])
        return out


class ReLU(Module):
    """nn.js:547."""

    def forward(self, x):
        return x.relu()


class Sequential(Module):
    """nn.js:560-569."""

    def __init__(self, *layers):
        super().__init__()
        for i, layer in enumerate(layers):
            self._modules[str(i)] = layer

    def forward(self, x):
        for m in self._modules.values():
            x = m.forward(x)
        return x
