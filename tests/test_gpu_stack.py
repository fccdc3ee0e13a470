"""Config 5 at its layer shape: the 4-layer stack (pre-RMSNorm -> SPARC -> residual per layer,
default init under torch.manual_seed(0), bfloat16 activations, float32 parameters) at width
2048, forward and backward on the GPU, against the float64 oracle's composition of
block_forward / block_backward (oracle/sparc_oracle.py) on the same bfloat16 input, with the
activations and gradients between layers rounded to bfloat16 as the stack's own are. The batch and
length are reduced (B=2, T=2048) so the float64 oracle finishes in seconds; every kernel runs at
the config's width and dtype. Tolerance: bfloat16 activations, 2e-2 relative l2 per tensor, or
1.5x the reference's own bfloat16 error where that is larger: its bf16 path misses float64 by
3.2e-2 on x.grad and phase_direction.grad and 3.3e-2 on radial_direction.grad (measured at the
config-2 layer, SPARCMixer(512), B=8, T=2048), which these sums over B x T tokens share."""
import numpy as np
import pytest
import torch

from oracle import sparc_oracle as O

pytestmark = pytest.mark.gpu

TOL = 2e-2
# 1.5x the reference's own bfloat16 error where that exceeds the bound
TOL_REF = {"phase_direction": 1.5 * 3.2e-2, "radial_direction": 1.5 * 3.3e-2, "x": 1.5 * 3.2e-2}


def test_config5_stack_matches_oracle_composition():
    from sparc_b200 import SPARCStack

    B, T, W, layers = 2, 2048, 2048, 4
    torch.manual_seed(0)
    stack = SPARCStack(W, layers).cuda()
    gen = torch.Generator(device="cuda").manual_seed(5)
    with torch.no_grad():  # live controllers and norm weights, so every gradient term is exercised
        for i in range(layers):
            m = stack.mixers[i]
            m.phase_direction.copy_(torch.randn(W + 1, generator=gen, device="cuda") / W ** 0.5)
            m.radial_direction.copy_(torch.randn(W + 1, generator=gen, device="cuda") / W ** 0.5)
            m.write_phase_response.copy_(torch.randn(W // 2, generator=gen, device="cuda") * 0.5)
            m.write_radial_response.copy_(torch.randn(W // 2, generator=gen, device="cuda") * 0.5)
            stack.norms[i].weight.copy_(1.0 + 0.1 * torch.randn(W, generator=gen, device="cuda"))
    x = torch.randn(B, T, W, generator=gen, device="cuda").to(torch.bfloat16).requires_grad_(True)
    g = torch.randn(B, T, W, generator=gen, device="cuda").to(torch.bfloat16)
    out = stack(x)
    out.backward(g)

    # the oracle: forward through the layers in float64 keeping each layer's input, then back;
    # the activations and gradients passed between layers are rounded to bfloat16 as the
    # stack's own are (bfloat16 activations), so each layer is compared on identical inputs
    def bf16(a):
        return torch.from_numpy(a).to(torch.bfloat16).double().numpy()

    xs = [x.detach().double().cpu().numpy()]
    Ps, ws = [], []
    for i in range(layers):
        m = stack.mixers[i]
        Ps.append(O.Params.from_mapping({k: getattr(m, k).detach().double().cpu().numpy() for k in O.PARAM_NAMES}))
        ws.append(stack.norms[i].weight.detach().double().cpu().numpy())
        y, _ = O.block_forward(xs[-1], Ps[-1], ws[-1])
        xs.append(bf16(y))
    assert O.rel_l2(out.detach().double().cpu().numpy(), xs[-1]) < TOL
    d = g.double().cpu().numpy()
    for i in reversed(range(layers)):
        gr = O.block_backward(xs[i], Ps[i], ws[i], d)
        m = stack.mixers[i]
        for k in [n for n in O.PARAM_NAMES if n != "energy_response"]:
            e = O.rel_l2(getattr(m, k).grad.double().cpu().numpy(), gr[k])
            assert e < TOL_REF.get(k, TOL), (i, k, e)
        e = O.rel_l2(stack.norms[i].weight.grad.double().cpu().numpy(), gr["norm_weight"])
        assert e < TOL, (i, "norm_weight", e)
        d = bf16(gr["x"]) if i > 0 else gr["x"]
    e = O.rel_l2(x.grad.double().cpu().numpy(), d)
    assert e < TOL_REF["x"], ("x", e)
    assert np.all(stack.mixers[0].energy_response.grad.cpu().numpy() == 0)
