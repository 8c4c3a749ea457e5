"""Pin the CPU oracle (the plain-C restatement) against the reference's own code and against the
golden vectors that reference build produced. CPU only."""
import os

import numpy as np
import pytest

import oracle as O
from roaster_b200 import synth
from tests.golden import make_golden as G

GOLD = os.path.join(os.path.dirname(__file__), "golden")
needs_ref = pytest.mark.skipif(not O.have_ref(), reason="reference build (oracle/_ref) absent")


def load(name):
    return np.load(os.path.join(GOLD, name))


def test_f16_rounding_matches_numpy(oracle_lib):
    lib = O._load("port")
    vals = np.array([0.0, -0.0, 1.0, -2.5, 65504.0, 65519.9, 65520.0, 1e-8, 6e-8, 3e-5,
                     6.1035e-05, 0.1, 1 / 3, np.inf, -np.inf, 2049.0, 2051.0, 4097.0],
                    np.float32)
    rng = np.random.default_rng(3)
    vals = np.concatenate([vals, rng.standard_normal(2000).astype(np.float32) * 100,
                           rng.standard_normal(2000).astype(np.float32) * 1e-5])
    mine = np.array([lib.orc_f32_to_f16(float(v)) for v in vals], np.uint16)
    ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(mine, ref)


def test_golden_decode_cfg0(oracle_lib):
    g = load("attn_decode_cfg0.npz")
    d, dg = G.decode_case()
    assert dg == str(g["digest"]), "synthetic input generator changed"
    out, ka, va = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"],
                                d["k_norm"], d["k_cache"], d["v_cache"], 512, 512)
    assert O.maxrel(out, g["out"]) < 1e-5
    assert O.maxrel(ka, g["k_app"]) < 1e-5
    assert np.array_equal(va, g["v_app"])


def test_golden_delta_16_steps(oracle_lib):
    g = load("delta_16steps.npz")
    state, seq, dg = G.delta_case()
    assert dg == str(g["digest"])
    st = state.copy()
    outs = [O.delta_step(st, seq["q"][t, 0], seq["k"][t, 0], seq["v"][t, 0], seq["g"][t, 0],
                         seq["beta"][t, 0]) for t in range(16)]
    assert O.maxrel(outs[0], g["out_first"]) < 1e-6
    assert O.maxrel(outs[-1], g["out_last"]) < 1e-6
    assert O.maxrel(st[[0, 31]], g["state_heads_0_31"]) < 1e-6
    assert abs(st.astype(np.float64).sum() - float(g["state_sum"])) < 1e-3


def test_golden_prefill_t12(oracle_lib):
    g = load("attn_prefill_t12.npz")
    d, dg = G.prefill_case()
    assert dg == str(g["digest"])
    out, ka, va = O.attn_prefill(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"],
                                 d["k_cache"], d["v_cache"], 50, 300)
    assert O.maxrel(out, g["out"]) < 1e-5
    assert O.maxrel(ka, g["k_app"]) < 1e-5


@needs_ref
@pytest.mark.parametrize("length,position", [(0, 0), (1, 1), (37, 1000), (512, 512), (700, 262143)])
def test_port_vs_reference_decode(oracle_lib, length, position):
    d = synth.attn_decode_inputs(seed=length + 5, length=length, position=position)
    a = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                      d["k_cache"], d["v_cache"], length, position, impl="port")
    b = O.attn_decode(d["q"], d["gate"], d["k_new"], d["v_new"], d["q_norm"], d["k_norm"],
                      d["k_cache"], d["v_cache"], length, position, impl="ref")
    for x, y in zip(a, b):
        assert O.maxrel(x, y) < 1e-5


@needs_ref
def test_port_vs_reference_prefill_two_chunks(oracle_lib):
    # 300 tokens: the reference runs them as two pf_attention chunks (256 + 44).
    d = synth.prefill_inputs(seed=9, T=300, kbase=20)
    a = O.attn_prefill(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"], d["k_cache"],
                       d["v_cache"], 20, 20, impl="port")
    b = O.attn_prefill(d["q"], d["gate"], d["k"], d["v"], d["q_norm"], d["k_norm"], d["k_cache"],
                       d["v_cache"], 20, 20, impl="ref")
    for x, y in zip(a, b):
        assert O.maxrel(x, y) < 1e-5


@needs_ref
def test_port_vs_reference_delta(oracle_lib):
    st = synth.delta_state(4, 1)[0]
    st2 = st.copy()
    seq = synth.delta_sequence(5, 40, 1)
    a = O.delta_prefill(st, seq["q"][:, 0], seq["k"][:, 0], seq["v"][:, 0], seq["g"][:, 0],
                        seq["beta"][:, 0], impl="port")
    b = O.delta_prefill(st2, seq["q"][:, 0], seq["k"][:, 0], seq["v"][:, 0], seq["g"][:, 0],
                        seq["beta"][:, 0], impl="ref")
    assert np.array_equal(a, b)
    assert np.array_equal(st, st2)


def test_partial_merge_identity(oracle_lib):
    """Merging softmax partials of window slices equals attention over the whole window."""
    d = synth.attn_decode_inputs(seed=7, length=900)
    full = O.attn_decode_partial(d["q"], d["q_norm"], d["k_cache"], d["v_cache"], 0, 900, 900)
    parts = [O.attn_decode_partial(d["q"], d["q_norm"], d["k_cache"], d["v_cache"], a, b, 900)
             for a, b in ((0, 300), (300, 650), (650, 900))]
    M = np.max([p[0] for p in parts], axis=0)
    w = [p[1] * np.exp(p[0] - M) for p in parts]
    o = sum(wi[:, None] * p[2] for wi, p in zip(w, parts)) / sum(w)[:, None]
    assert O.maxrel(o, full[2]) < 1e-5


@pytest.mark.parametrize("T", [1, 2, 7, 70])
def test_port_vs_reference_delta_layer(oracle_lib, T):
    """The oracle's pre-ops + recurrence + gated RMSNorm equal the reference's own pf_ssm
    (model.c:1604-1660, driven with one-hot f32 projections) bit for bit."""
    if not O.have_ref():
        pytest.skip("reference build (oracle/_ref) not present")
    d = synth.delta_layer_inputs(10 + T, T)
    st0 = synth.delta_state(11, 1)[0]
    s1, c1 = st0.copy(), d["conv_state"].copy()
    s2, c2 = st0.copy(), d["conv_state"].copy()
    args = (d["qkv"], d["z"], d["alpha"], d["beta"], d["conv_w"], d["dt"], d["a"], d["ssm_norm"])
    a = O.delta_layer(s1, c1, *args, impl="port")
    b = O.delta_layer(s2, c2, *args, impl="ref")
    assert np.array_equal(a, b)
    assert np.array_equal(s1, s2)
    assert np.array_equal(c1, c2)


@pytest.mark.parametrize("q6", [False, True])
@pytest.mark.parametrize("rows,cols", [(1, 256), (300, 2048), (33, 4096)])
def test_port_vs_reference_matvec_q(oracle_lib, q6, rows, cols):
    """The oracle's Q4_K / Q6_K matvec against the reference's own kernel_dot_q4_k /
    kernel_dot_q6_k per row (matvec_q4_cpu / matvec_q6_cpu): fp32 sums in a different order,
    so 2e-6 maxrel rather than bit equality."""
    if not O.have_ref():
        pytest.skip("reference build (oracle/_ref) not present")
    m = synth.quant_matrix(rows + cols, rows, cols, q6)
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    a = O.matvec_q(q6, m, x, rows, cols, impl="port")
    b = O.matvec_q(q6, m, x, rows, cols, impl="ref")
    assert O.maxrel(a, b) < 2e-6


@pytest.mark.parametrize("q6", [False, True])
@pytest.mark.parametrize("rows,cols,T", [(37, 2048, 3), (300, 512, 40), (64, 4096, 257)])
def test_port_vs_reference_matmul_q(oracle_lib, q6, rows, cols, T):
    """The oracle's per-token matvec against the reference's own CPU prefill matmul
    (matmul_quant_cpu: dequantise a block to fp32, then dot it with each token; more than 256
    tokens run as 256-token chunks). Same fp32 terms summed in another order: 2e-6 maxrel."""
    if not O.have_ref():
        pytest.skip("reference build (oracle/_ref) not present")
    m = synth.quant_matrix(rows + T, rows, cols, q6)
    X = np.random.default_rng(T).standard_normal((T, cols)).astype(np.float32)
    a = O.matmul_q(q6, m, X, rows, cols, impl="port")
    b = O.matmul_q(q6, m, X, rows, cols, impl="ref")
    assert O.maxrel(a, b) < 2e-6
