"""The reference README's two usage examples (sparc-kernal/README.md: sequence training, then
single-step decoding from the returned cache), run as written against sparc_b200.SPARCMixer, with
checks: shapes and dtypes as the README states them, finite gradients, and the decode step
continuing the sequence (its output equals the last token of the sequence over prompt + input,
to bfloat16 rounding)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_readme_sequence_training_and_decoding():
    from sparc_b200 import SPARCMixer

    torch.manual_seed(0)
    # Sequence training
    x = torch.randn(2, 128, 128, device="cuda", dtype=torch.bfloat16)
    module = SPARCMixer(128).cuda().train()
    output, _ = module(x)
    loss = output.float().square().mean()
    loss.backward()
    assert output.shape == (2, 128, 128) and output.dtype == torch.bfloat16
    for n in ("nu_log", "theta_log", "phase_direction", "radial_direction", "write_log_gain",
              "write_phase_response", "write_radial_response"):
        g = getattr(module, n).grad
        assert g is not None and bool(torch.isfinite(g).all()), n

    # Single-step decoding
    module.eval()
    with torch.no_grad():
        prompt = torch.randn(2, 128, 128, device="cuda", dtype=torch.bfloat16)
        _, state = module(prompt, return_cache=True)

        module.prepare_inference()
        next_input = torch.randn(2, 128, device="cuda", dtype=torch.bfloat16)
        next_output, state = module.step(next_input, state, segment_pos=None)

        assert next_output.shape == (2, 128) and next_output.dtype == torch.bfloat16
        assert state[0].shape == (2, 64) and state[0].dtype == torch.float32 and state[1].shape == (2, 64)
        full, last = module(torch.cat((prompt, next_input[:, None]), dim=1), return_cache=True)
        assert torch.allclose(next_output.float(), full[:, -1].float(), rtol=2e-2, atol=2e-2)
        assert torch.allclose(state[0], last[0], rtol=1e-2, atol=1e-2)
        assert torch.allclose(state[1], last[1], rtol=1e-2, atol=1e-2)
