"""Precision budget of the chunked DeltaNet prefill's f16 tensor-core products (CPU).

deltanet_prefill_kernel regroups the reference's sequential recurrence (model.c:1507-1534, as
pf_ssm runs it, model.c:1644-1658) into chunks of 64 tokens and runs every product on f16
tensor cores as three terms, hi*hi + hi*lo + lo*hi, with hi = f16(x) and lo = f16(x - hi)
after a power-of-two row scale. This file emulates that chunked form in float64 with each
product's operands rounded the same way, and checks it against the oracle's fp32 sequential
recurrence at 2048 tokens with the bar of the GPU tests (maxrel 1e-4 on state and outputs):

- three terms everywhere pass with a wide margin;
- one f16 term everywhere, or two terms everywhere, fail;
- W = T diag(beta e^G) K and W S_0 tolerate two terms (T and W the single-term operands);
  Q K^T and the state update K^T Delta do not.

Dropping those two terms removes about 1.05 of the 34.6 MFLOP the tensor pipe executes per
(chunk, value head), 3 %, which is why the kernel keeps three terms throughout."""
import numpy as np
import pytest

import oracle as O
from roaster_b200 import synth

T_TOKENS, HEADS, CHUNK, TOL = 2048, 8, 64, 1e-4


def _split(x):
    """hi/lo f16 parts of x with a power-of-two scale per row (last axis)."""
    m = np.abs(x).max(axis=-1, keepdims=True)
    e = np.where(m > 0, np.floor(np.log2(np.where(m > 0, m, 1.0))) + 1, 0).astype(int)
    y = x * np.ldexp(1.0, -e)
    hi = y.astype(np.float16).astype(np.float64)
    lo = (y - hi).astype(np.float16).astype(np.float64)
    return hi * np.ldexp(1.0, e), lo * np.ldexp(1.0, e)


def _mm(a, b, terms):
    """a @ b from f16 parts: "3" = hi.hi + hi.lo + lo.hi; "1" = hi.hi; "2a" keeps a's lo
    (b single f16); "2b" keeps b's lo (a single f16)."""
    ah, al = _split(a)
    bh, bl = (np.swapaxes(t, -1, -2) for t in _split(np.swapaxes(b, -1, -2)))
    r = ah @ bh
    if terms in ("3", "2b"):
        r = r + ah @ bl
    if terms in ("3", "2a"):
        r = r + al @ bh
    return r


def _chunked(p, st0, modes):
    """The kernel's chunked regrouping with per-product term counts; returns (state, out)."""
    S = st0[:HEADS].astype(np.float64)                              # [H, dk, dv]
    kh = np.arange(HEADS) % 16                                      # value head vh reads key head vh % 16
    T = p["q"].shape[0]
    out = np.zeros((T, HEADS, 128))
    mm = lambda a, b, name: _mm(a, b, modes.get(name, "3"))        # noqa: E731
    for c0 in range(0, T, CHUNK):
        c1 = min(T, c0 + CHUNK)
        n = c1 - c0
        Q, K = (p[x][c0:c1, kh].transpose(1, 0, 2).astype(np.float64) for x in ("q", "k"))
        V = p["v"][c0:c1, :HEADS].transpose(1, 0, 2).astype(np.float64)
        g, b = (p[x][c0:c1, :HEADS].T.astype(np.float64) for x in ("g", "beta"))
        G = np.cumsum(g, axis=1)
        gam = np.exp(G)
        E = np.exp(G[:, :, None] - G[:, None, :])
        L = b[:, :, None] * E * mm(K, np.swapaxes(K, 1, 2), "KK") * np.tril(np.ones((n, n)), -1)
        Tm = np.linalg.inv(np.eye(n)[None] + L)
        U = mm(Tm, b[:, :, None] * V, "U")
        W = mm(Tm, (b * gam)[:, :, None] * K, "W")
        D = U - mm(W, S, "WS")
        M = E * mm(Q, np.swapaxes(K, 1, 2), "QK") * np.tril(np.ones((n, n)), 0)
        out[c0:c1] = ((mm(gam[:, :, None] * Q, S, "QS") + mm(M, D, "MD")) / np.sqrt(128.0)).transpose(1, 0, 2)
        w = np.exp(G[:, -1:] - G)
        S = gam[:, -1][:, None, None] * S + mm(np.swapaxes(K, 1, 2), w[:, :, None] * D, "SU")
    return S, out


@pytest.fixture(scope="module")
def case(oracle_lib):
    p = synth.delta_prompt(41, T_TOKENS)
    st0 = synth.delta_state(42, 1)[0]
    st = st0.copy()
    out = O.delta_prefill(st, p["q"], p["k"], p["v"], p["g"], p["beta"])
    return p, st0, st[:HEADS], out[:, :HEADS]


ALL = ("KK", "QK", "U", "W", "WS", "QS", "MD", "SU")


def _err(case, modes):
    p, st0, st_ref, out_ref = case
    S, out = _chunked(p, st0, modes)
    return O.maxrel(S, st_ref), O.maxrel(out, out_ref)


def test_three_terms_everywhere_pass_with_margin(case):
    s, o = _err(case, {})
    assert s < 1e-6 and o < 1e-6


@pytest.mark.parametrize("terms", ["1", "2a"])
def test_fewer_terms_everywhere_fail(case, terms):
    s, o = _err(case, {k: terms for k in ALL})
    assert max(s, o) > TOL


def test_w_products_tolerate_two_terms(case):
    s, o = _err(case, {"W": "2b", "WS": "2b"})
    assert s < TOL and o < TOL / 4


@pytest.mark.parametrize("name", ["QK", "SU"])
def test_score_and_state_update_need_three_terms(case, name):
    s, o = _err(case, {name: "2b"})
    assert max(s, o) > TOL
