"""CPU tests of the Python entry point and the operator registration:
argument checks with the reference's exception types (ops.py:13-22 of the
reference), the torch op schema and the FakeTensor kernel (_loader.py:41-48)."""
from __future__ import annotations

import pytest
import torch

import muon_ascend950
import muon_fusion_ascend950_b200 as pkg


def test_drop_in_alias():
    assert muon_ascend950.polar_step is pkg.polar_step
    assert pkg.__version__ == "0.1.1"


def test_drop_in_alias_submodules():
    """The reference's module paths (muon_ascend950/ops.py, _loader.py)
    resolve to this build's modules of the same role."""
    import importlib

    ops = importlib.import_module("muon_ascend950.ops")
    loader = importlib.import_module("muon_ascend950._loader")
    assert ops is pkg.ops and ops.polar_step is pkg.polar_step
    assert loader.load_library is pkg.load_library
    from muon_ascend950.ops import polar_step  # noqa: F401  (the reference's import form)


def test_rejects_non_tensor():
    with pytest.raises(TypeError):
        pkg.polar_step([[1.0]], 1.0, 1.0, 1.0)


def test_rejects_cpu_tensor():
    with pytest.raises(ValueError):
        pkg.polar_step(torch.zeros(4, 8, dtype=torch.bfloat16), 1.0, 1.0, 1.0)


def test_rejects_meta_device():
    with pytest.raises(ValueError):
        pkg.polar_step(torch.zeros(4, 8, dtype=torch.bfloat16, device="meta"), 1.0, 1.0, 1.0)


def test_op_schema():
    schema = str(torch.ops.muon_ascend950.polar_step.default._schema)
    assert schema == "muon_ascend950::polar_step(Tensor x, float a, float b, float c) -> Tensor"


@pytest.mark.parametrize("shape", [(2, 4, 8), (1, 129, 130)])
def test_fake_tensor_kernel(shape):
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        x = torch.empty(shape, dtype=torch.bfloat16, device="cuda")
        y = torch.ops.muon_ascend950.polar_step(x, 1.0, 2.0, 3.0)
        assert y.shape == x.shape and y.dtype == x.dtype and y.is_contiguous()


def test_loader_respects_library_override(tmp_path, monkeypatch):
    from muon_fusion_ascend950_b200 import _loader

    monkeypatch.setenv("MUON_ASCEND950_LIBRARY", str(tmp_path / "missing.so"))
    with pytest.raises(RuntimeError, match="does not exist"):
        _loader._library_path()


def test_fake_kernel_traces_into_a_graph():
    """The operator traces through the FakeTensor kernel (no device needed):
    make_fx in fake mode records one call of the op with the input's shape."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def f(x):
        return torch.ops.muon_ascend950.polar_step(x, 1.5, -0.5, 0.25)

    gm = make_fx(f, tracing_mode="fake")(torch.empty(2, 16, 32, dtype=torch.bfloat16))
    calls = [n for n in gm.graph.nodes if n.op == "call_function"]
    assert [str(n.target) for n in calls] == ["muon_ascend950.polar_step.default"]
    assert tuple(calls[0].meta["val"].shape) == (2, 16, 32)


def test_fake_kernel_of_the_transposed_op():
    """polar_step_t (tall X in its own layout) has the same FakeTensor
    contract as polar_step."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def f(x):
        return torch.ops.muon_ascend950.polar_step_t(x, 1.5, -0.5, 0.25)

    gm = make_fx(f, tracing_mode="fake")(torch.empty(2, 48, 16, dtype=torch.bfloat16))
    calls = [n for n in gm.graph.nodes if n.op == "call_function"]
    assert [str(n.target) for n in calls] == ["muon_ascend950.polar_step_t.default"]
    assert tuple(calls[0].meta["val"].shape) == (2, 48, 16)


def test_fake_kernels_of_the_caller_side_ops():
    """polar_express returns bf16 of x's shape; muon_update_ mutates and
    returns nothing: both trace in fake mode."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def f(x):
        return torch.ops.muon_ascend950.polar_express(x, [1.0, 0.5, 0.25] * 2, True)

    gm = make_fx(f, tracing_mode="fake")(torch.empty(2, 16, 32, dtype=torch.float32))
    call = [n for n in gm.graph.nodes if n.op == "call_function"][0]
    assert call.meta["val"].dtype == torch.bfloat16
    assert tuple(call.meta["val"].shape) == (2, 16, 32)

    def g(p, grad, buf):
        torch.ops.muon_ascend950.muon_update_(p, grad, buf, 0.02, 0.95, True, 0.0, 1.0,
                                              [1.0, 0.5, 0.25])
        return p

    t = torch.empty(16, 32)
    gm = make_fx(g, tracing_mode="fake")(t, t.clone(), t.clone())
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert "muon_ascend950.muon_update_.default" in targets


def test_muon_optimizer_argument_checks():
    import muon_fusion_ascend950_b200 as pkg

    w = torch.nn.Parameter(torch.zeros(4, 4))
    with pytest.raises(ValueError):
        pkg.Muon([w], lr=-1.0)
    with pytest.raises(ValueError):
        pkg.Muon([w], momentum=1.0)
    with pytest.raises(ValueError):
        pkg.Muon([w], coefficients=[(1.0, 2.0)])
    v = torch.nn.Parameter(torch.zeros(4))
    opt = pkg.Muon([v])
    v.grad = torch.zeros(4)
    with pytest.raises(ValueError, match="matrices"):
        opt.step()


def test_polar_express_argument_checks():
    import muon_fusion_ascend950_b200 as pkg

    with pytest.raises(TypeError):
        pkg.polar_express([1.0])
    with pytest.raises(ValueError):
        pkg.polar_express(torch.zeros(2, 3, dtype=torch.bfloat16))  # not on CUDA
