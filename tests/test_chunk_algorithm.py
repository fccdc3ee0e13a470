"""The decomposition the mixer kernels implement, restated in float64 numpy and checked against the
serial scan and its adjoint for random shapes (hypothesis): per chunk the affine map
h_out = P h_in + Q (P the product of the chunk's transitions, Q the chunk run from zero), the
chunk carries composed span by span in a fixed order (CTA q of the carry scan composes its span
of chunks, then the earlier spans' maps in order), and the replay of every chunk from its
carried-in state; the backward mirrors it with reverse maps of the adjoint
lambda_t = g_t + conj(a_{t+1}) lambda_{t+1}. Resets zero a_t, so a chunk map across a reset has
P = 0 and the composition needs nothing special; h0 enters as the carry into the first chunk."""
import numpy as np
from hypothesis import given, settings
from hypothesis import strategies as st


def _serial(a, b, h0):
    B, T, M = b.shape
    h = h0.copy()
    out = np.empty_like(b)
    for t in range(T):
        h = a[:, t] * h + b[:, t]
        out[:, t] = h
    return out


def _serial_adjoint(a, g, gl):
    """lambda_t = g_t + conj(a_{t+1}) lambda_{t+1}, lambda_{T-1} = g_{T-1} + grad_last; returns
    lambda and the gradient of h0 (conj(a_0) lambda_0)."""
    B, T, M = g.shape
    lam = gl.copy()
    out = np.empty_like(g)
    for t in range(T - 1, -1, -1):
        lam = lam + g[:, t]
        out[:, t] = lam
        lam = np.conj(a[:, t]) * lam
    return out, lam


def _chunked(a, b, h0, C, q):
    """summary -> carry scan (spans of q chunks) -> replay."""
    B, T, M = b.shape
    n = -(-T // C)
    P = np.ones((B, n, M), complex)
    Q = np.zeros((B, n, M), complex)
    for k in range(n):  # summary: the chunk's map from a zero state
        for t in range(k * C, min(T, (k + 1) * C)):
            P[:, k] = a[:, t] * P[:, k]
            Q[:, k] = a[:, t] * Q[:, k] + b[:, t]
    carry_in = np.empty((B, n, M), complex)
    spans = [list(range(s, min(n, s + q))) for s in range(0, n, q)]
    span_maps = []
    for sp in spans:  # each span's composed map, independently
        SP, SQ = np.ones((B, M), complex), np.zeros((B, M), complex)
        for k in sp:
            SP, SQ = P[:, k] * SP, P[:, k] * SQ + Q[:, k]
        span_maps.append((SP, SQ))
    for i, sp in enumerate(spans):  # earlier spans composed in order, then the span's own chunks
        h = h0.copy()
        for SP, SQ in span_maps[:i]:
            h = SP * h + SQ
        for k in sp:
            carry_in[:, k] = h
            h = P[:, k] * h + Q[:, k]
    out = np.empty_like(b)
    for k in range(n):  # replay
        h = carry_in[:, k]
        for t in range(k * C, min(T, (k + 1) * C)):
            h = a[:, t] * h + b[:, t]
            out[:, t] = h
    return out, h


def _chunked_adjoint(a, g, gl, C, q):
    """The backward's reverse summary (each chunk's map from the adjoint arriving at its last
    token to the adjoint at its first token, R lambda + S), the reverse carry scan and the replay
    of the true adjoint; returns lambda and the gradient of h0."""
    B, T, M = g.shape
    n = -(-T // C)
    R = np.ones((B, n, M), complex)
    S = np.zeros((B, n, M), complex)
    for k in range(n):
        for t in range(min(T, (k + 1) * C) - 1, k * C - 1, -1):
            # lambda_t = g_t + conj(a_{t+1}) lambda_{t+1} inside the chunk
            S[:, k] = S[:, k] + g[:, t]
            if t > k * C:
                R[:, k] = np.conj(a[:, t]) * R[:, k]
                S[:, k] = np.conj(a[:, t]) * S[:, k]
    # the whole chunk as a map from the adjoint arriving at its last token to the one leaving it
    # (conj(a) of its first token applied): RR lam + SS; the reverse carry scan composes these
    # maps span by span, from the last span backwards, in a fixed order
    RR = np.conj(a[:, 0:T:C]) * R
    SS = np.conj(a[:, 0:T:C]) * S
    carry = np.empty((B, n, M), complex)  # adjoint arriving at the last token of chunk k
    spans = [list(range(s, max(-1, s - q), -1)) for s in range(n - 1, -1, -q)]
    span_maps = []
    for sp in spans:
        SP, SQ = np.ones((B, M), complex), np.zeros((B, M), complex)
        for k in sp:
            SP, SQ = RR[:, k] * SP, RR[:, k] * SQ + SS[:, k]
        span_maps.append((SP, SQ))
    for i, sp in enumerate(spans):
        lam_next = gl.copy()
        for SP, SQ in span_maps[:i]:
            lam_next = SP * lam_next + SQ
        for k in sp:
            carry[:, k] = lam_next
            lam_next = RR[:, k] * lam_next + SS[:, k]
    out = np.empty_like(g)
    for k in range(n):
        lam = carry[:, k]
        for t in range(min(T, (k + 1) * C) - 1, k * C - 1, -1):
            lam = lam + g[:, t]
            out[:, t] = lam
            lam = np.conj(a[:, t]) * lam
    return out, lam_next


@settings(max_examples=60, deadline=None)
@given(B=st.integers(1, 3), T=st.integers(1, 70), M=st.integers(1, 5), C=st.sampled_from([1, 2, 8, 16]),
       q=st.integers(1, 5), resets=st.integers(0, 4), seed=st.integers(0, 2 ** 16))
def test_chunk_decomposition_equals_serial_scan(B, T, M, C, q, resets, seed):
    rng = np.random.default_rng(seed)
    rho = rng.uniform(0.3, 0.999, (B, T, M))
    a = rho * np.exp(1j * rng.uniform(-np.pi, np.pi, (B, T, M)))
    for _ in range(resets):  # a reset zeroes the token's transition
        a[rng.integers(B), rng.integers(T)] = 0.0
    b = rng.standard_normal((B, T, M)) + 1j * rng.standard_normal((B, T, M))
    h0 = rng.standard_normal((B, M)) + 1j * rng.standard_normal((B, M))
    ref = _serial(a, b, h0)
    out, last = _chunked(a, b, h0, C, q)
    assert np.allclose(out, ref, rtol=1e-10, atol=1e-10) and np.allclose(last, ref[:, -1], rtol=1e-10, atol=1e-10)
    g = rng.standard_normal((B, T, M)) + 1j * rng.standard_normal((B, T, M))
    gl = rng.standard_normal((B, M)) + 1j * rng.standard_normal((B, M))
    lam_ref, gh0_ref = _serial_adjoint(a, g, gl)
    lam, gh0 = _chunked_adjoint(a, g, gl, C, q)
    assert np.allclose(lam, lam_ref, rtol=1e-10, atol=1e-10) and np.allclose(gh0, gh0_ref, rtol=1e-10, atol=1e-10)
