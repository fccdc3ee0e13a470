"""The torch.ops.sparc_b200 operators under tracing, without a GPU: their fake kernels give the
C++ operators' output shapes and dtypes (from the library's host-only queries), autograd runs
through the registered formulas (mixer_forward -> mixer_backward, real_scan_forward ->
real_scan_backward) on fake tensors, make_fx traces them with symbolic shapes, and
torch.compile captures a full graph with them (a recording backend; nothing is executed)."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

PARAMS = ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
          "write_phase_response", "write_radial_response")


@pytest.fixture(scope="module")
def ops():
    from sparc_b200 import _build, torch_ops

    _build.build()
    _build.build_torch_ops()
    return torch_ops.load()


def _params(W, device, requires_grad=False):
    M = W // 2
    sizes = {"phase_direction": W + 1, "radial_direction": W + 1}
    return [torch.randn(sizes.get(n, M), device=device, requires_grad=requires_grad) for n in PARAMS]


@pytest.mark.parametrize("dtype,T", [(torch.float32, 37), (torch.bfloat16, 64), (torch.float32, 1)])
def test_fake_shapes(ops, dtype, T):
    from sparc_b200 import _lib

    L = _lib.lib()
    B, W = 3, 10
    M = W // 2
    dt = _lib.dtype_code(dtype)
    with FakeTensorMode():
        x = torch.randn(B, T, W, device="cuda").to(dtype)
        p = _params(W, "cuda")
        y, lr, li, carry, ctl, st = ops.mixer_forward(x, *p)
        assert y.shape == x.shape and y.dtype == dtype and y.device == x.device
        assert lr.shape == li.shape == (B, M) and lr.dtype == torch.float32
        assert carry.shape == (B, L.sparc_mixer_carry_chunks(T, dt), M, 2)
        assert ctl.shape == (B, T, L.sparc_mixer_controls_floats())
        assert st.shape == x.shape and st.dtype == dtype
        g = ops.mixer_backward(x, y, y, *p, carry, ctl, st)
        assert [t.shape for t in g] == [x.shape] + [(n,) for n in (M, M, W + 1, W + 1, M, M, M, M)]
        yd, nr, ni = ops.decode_step(x[:, 0], lr, li, *p)
        assert yd.shape == (B, W) and yd.dtype == dtype and nr.shape == ni.shape == (B, M)
        a = torch.rand(B, T, 7, device="cuda").to(dtype)
        out, rc, last = ops.real_scan_forward(a, a)
        assert out.shape == a.shape and out.dtype == dtype
        assert rc.shape == (B, L.sparc_real_carry_chunks(T), 7) and last.shape == (B, 7)
        ga, gb = ops.real_scan_backward(a, a, out, rc)
        assert ga.shape == gb.shape == a.shape


def test_autograd_through_the_operators(ops):
    # (fake tensors on the CPU device: the autograd engine would open a CUDA context for fake
    # CUDA tensors, and this box has no GPU; the fake kernels do not depend on the device)
    B, T, W = 2, 19, 12
    with FakeTensorMode():
        x = torch.randn(B, T, W, requires_grad=True)
        p = _params(W, "cpu", requires_grad=True)
        y, lr, li, carry, ctl, st = ops.mixer_forward(x, *p)
        assert y.requires_grad and not lr.requires_grad and not carry.requires_grad and not ctl.requires_grad
        assert not st.requires_grad
        (y * y).sum().backward()
        assert x.grad is not None and x.grad.shape == x.shape
        for t in p:
            assert t.grad is not None and t.grad.shape == t.shape and t.grad.dtype == torch.float32
        a = torch.rand(B, T, 5, requires_grad=True)
        b = torch.randn(B, T, 5, requires_grad=True)
        out, carry, last = ops.real_scan_forward(a, b)
        assert out.requires_grad and not carry.requires_grad and not last.requires_grad
        out.sum().backward()
        assert a.grad.shape == a.shape and b.grad.shape == b.shape


def test_make_fx_symbolic(ops):
    from torch.fx.experimental.proxy_tensor import make_fx

    def f(x, *p):
        y, lr, li, carry, ctl, st = torch.ops.sparc_b200.mixer_forward(x, *p)
        return y, carry

    # (real CPU inputs: make_fx fakes them with symbolic sizes and never runs a kernel)
    gm = make_fx(f, tracing_mode="symbolic")(torch.randn(2, 40, 8), *_params(8, "cpu"))
    calls = [n for n in gm.graph.nodes if n.op == "call_function" and "sparc_b200.mixer_forward" in str(n.target)]
    assert len(calls) == 1
    y, carry = [n.meta["val"] for n in gm.graph.output_node().args[0]]
    assert isinstance(y.shape[1], torch.SymInt) and isinstance(carry.shape[1], torch.SymInt)  # T and ceil(T / C)


def test_torch_compile_captures_a_full_graph(ops):
    seen = []

    def backend(gm, example_inputs):
        seen.append(gm)
        # record the graph only (no GPU here to run it): return placeholders of the outputs' shapes
        vals = [n.meta["example_value"] for n in gm.graph.output_node().args[0]]
        return lambda *args: [torch.zeros(v.shape, dtype=v.dtype) for v in vals]

    def f(a, b):
        out, carry, last = torch.ops.sparc_b200.real_scan_forward(a, b)
        return out * 2.0

    compiled = torch.compile(f, backend=backend, fullgraph=True)
    compiled(torch.rand(2, 32, 3), torch.rand(2, 32, 3))
    assert len(seen) == 1
    targets = [str(n.target) for n in seen[0].graph.nodes if n.op == "call_function"]
    assert any("sparc_b200.real_scan_forward" in t for t in targets)
