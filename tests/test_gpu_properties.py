"""Property tests: random small shapes against the oracle (hypothesis), linearity of the states
in the initial state (the projection variant's states have no relu), and invariance of the real
scan under the chunk size it is given (to rounding)."""
import numpy as np
import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu


@settings(max_examples=12, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(B=st.integers(1, 3), T=st.integers(1, 70), M=st.integers(1, 300), seed=st.integers(0, 2 ** 16))
def test_mixer_random_shapes_match_oracle(B, T, M, seed):
    import sparc_b200

    W = 2 * M
    torch.manual_seed(seed)
    m = sparc_b200.SPARCMixer(W).cuda()
    with torch.no_grad():
        m.phase_direction.normal_(0, 1.0 / W ** 0.5)
        m.radial_direction.normal_(0, 1.0 / W ** 0.5)
        m.write_phase_response.normal_(0, 0.5)
        m.write_radial_response.normal_(0, 0.5)
    x = torch.randn(B, T, W, device="cuda", requires_grad=True)
    g = torch.randn(B, T, W, device="cuda")
    y, _ = m(x)
    y.backward(g)
    P = O.Params.from_mapping({k: getattr(m, k).detach().double().cpu().numpy() for k in O.PARAM_NAMES})
    xd = x.detach().double().cpu().numpy()
    y_ref, _, _ = O.sparc_forward(xd, P)
    g_ref = O.sparc_backward(xd, P, g.double().cpu().numpy())
    assert O.rel_l2(y.detach().double().cpu().numpy(), y_ref) < 1e-4
    assert O.rel_l2(x.grad.double().cpu().numpy(), g_ref["x"]) < 1e-3
    for k in ("nu_log", "theta_log", "write_log_gain"):
        if np.abs(g_ref[k]).max() > 1e-8:
            assert O.rel_l2(getattr(m, k).grad.double().cpu().numpy(), g_ref[k]) < 1e-3, k


def test_projection_states_are_affine_in_the_initial_state():
    import sparc_b200

    B, T, W, M = 2, 60, 24, 40
    torch.manual_seed(1)
    layer = sparc_b200.SPARCSequenceLayer(W, M).cuda()
    params = {n: p.detach() for n, p in layer.named_parameters()}
    x = torch.randn(B, T, W, device="cuda")
    ha = (torch.randn(B, M, device="cuda"), torch.randn(B, M, device="cuda"))
    hb = (torch.randn(B, M, device="cuda"), torch.randn(B, M, device="cuda"))
    zero = (torch.zeros(B, M, device="cuda"), torch.zeros(B, M, device="cuda"))

    def states(h0):
        (hr, hi), _ = sparc_b200.sparc_projection_states(x, params, state=h0)
        return torch.cat((hr, hi), -1).double()

    s0 = states(zero)
    lhs = states((ha[0] + hb[0], ha[1] + hb[1])) - s0
    rhs = (states(ha) - s0) + (states(hb) - s0)
    assert float((lhs - rhs).norm() / rhs.norm()) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_real_chunk_scan_is_invariant_to_the_chunk(dtype):
    import sparc_b200

    a = (torch.rand(2, 256, 130, device="cuda") * 0.5 + 0.45).to(dtype)
    b = torch.randn(2, 256, 130, device="cuda").to(dtype)
    outs = [sparc_b200.real_chunk_scan(a, b, c).float() for c in (16, 32, 64, 128)]
    # (the decoupled lookback composes carries in an order that can differ run to run, so the
    # results agree to rounding: float32 ulps, or one bfloat16 ulp of the stored output)
    tol = dict(rtol=1e-5, atol=1e-6) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
    for o in outs[1:]:
        assert torch.allclose(o, outs[0], **tol)
