"""The PureAttention module exposes the reference's Python surface
(bindings.cpp:37-125): same classes, methods, argument names and defaults.
Runs without a GPU (only inspects the module)."""
import pytest


@pytest.fixture(scope="module")
def pa():
    import PureAttention
    return PureAttention


def test_reference_names_exist(pa):
    for name in ("Tensor", "Module", "Linear", "ReLU", "MultiheadAttention", "LayerNorm", "MSE",
                 "Adam", "fill_normal", "add"):
        assert hasattr(pa, name), name
    for meth in ("backward", "to_host", "to_device", "grad_to_host", "shape", "get_grad_stats"):
        assert hasattr(pa.Tensor, meth), meth
    assert hasattr(pa.Linear, "weight") and hasattr(pa.Linear, "bias")
    assert hasattr(pa.LayerNorm, "gamma") and hasattr(pa.LayerNorm, "beta")
    for meth in ("step", "zero_grad"):
        assert hasattr(pa.Adam, meth)
    assert hasattr(pa.MSE, "__call__")


def _default(doc, name):
    """Default value printed for argument `name` in a pybind11 signature line."""
    import re
    m = re.search(r"\b%s: [^=,]*(?:\[[^\]]*\][^=,]*)?= ([^,)]+)" % name, doc)
    return m.group(1).strip() if m else None


def test_argument_names_and_defaults(pa):
    assert _default(pa.Tensor.__init__.__doc__, "requires_grad") == "False"
    assert _default(pa.Tensor.backward.__doc__, "seed_with_ones") == "True"
    assert abs(float(_default(pa.LayerNorm.__init__.__doc__, "epsilon")) - 1e-5) < 1e-9
    doc = pa.Adam.__init__.__doc__
    for name, val in (("lr", 1e-3), ("beta1", 0.9), ("beta2", 0.999), ("eps", 1e-8)):
        assert abs(float(_default(doc, name)) - val) < 1e-6 * max(val, 1e-8), name
    assert float(_default(pa.fill_normal.__doc__, "std_dev")) == 1.0
    assert "params" in doc and "normalized_shape" in pa.LayerNorm.__init__.__doc__
    # both MultiheadAttention.forward overloads
    assert pa.MultiheadAttention.forward.__doc__.count("forward(") >= 2


def test_python_subclass_of_module(pa):
    class Twice(pa.Module):
        def __init__(self):
            super().__init__()

        def forward(self, x):
            return x

    m = Twice()
    assert m.parameters() == []
