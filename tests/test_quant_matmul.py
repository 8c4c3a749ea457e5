"""Multi-token k-quant projections (kernel_cuda_matmul_quant_batch) on the reference's own test
shapes (src/test_kernels.c:42-70: T in 1, 3, 8, 9, 16, 17, 100, 257; rows 512, 2048, 37; cols
2048 or 512; Q4_K and Q6_K; several jobs sharing X), against the reference's own CPU prefill
matmul (matmul_quant_cpu, kernels.c:1877-1913, built into oracle/_ref; the oracle restatement
token by token where that build is absent). Its own test bar is 2e-4 maxrel, this one 1e-5."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _ref(q6, m, X, rows, cols):
    return O.matmul_q(q6, m, X, rows, cols, impl="ref" if O.have_ref() else "port")


@pytest.mark.parametrize("q6", [False, True])
@pytest.mark.parametrize("rows,cols", [(512, 2048), (2048, 512), (37, 2048)])
@pytest.mark.parametrize("T", [1, 3, 8, 9, 16, 17, 100, 257])
def test_matmul(rb, oracle_lib, q6, rows, cols, T):
    m = synth.quant_matrix(rows * 7 + cols + int(q6), rows, cols, q6)
    X = np.random.default_rng(T + rows).uniform(-1, 1, (T, cols)).astype(np.float32)
    Y = torch.zeros(T, rows, device="cuda")
    rb.matmul_quant_batch([(q6, dev(m), dev(X), Y, rows, cols, T)])
    assert O.maxrel(host(Y), _ref(q6, m, X, rows, cols)) < TOL


def test_shared_x(rb, oracle_lib):
    """Three jobs sharing X in one call (the reference's shared-X case)."""
    T, cols = 40, 2048
    X = np.random.default_rng(5).uniform(-1, 1, (T, cols)).astype(np.float32)
    dX = dev(X)
    specs = [(False, 256), (True, 64), (False, 32)]
    keep, jobs, refs = [], [], []
    for i, (q6, r) in enumerate(specs):
        m = synth.quant_matrix(50 + i, r, cols, q6)
        dm, Y = dev(m), torch.zeros(T, r, device="cuda")
        keep.append((dm, Y))
        jobs.append((q6, dm, dX, Y, r, cols, T))
        refs.append(_ref(q6, m, X, r, cols))
    rb.matmul_quant_batch(jobs)
    for (dm, Y), ref in zip(keep, refs):
        assert O.maxrel(host(Y), ref) < TOL


def test_rejects_invalid(rb):
    m = torch.zeros(144, dtype=torch.uint8, device="cuda")
    X = torch.zeros(256, device="cuda")
    Y = torch.zeros(1, device="cuda")
    for bad in [(False, m, X, Y, 1, 300, 1), (False, m, X, Y, 1, 256, 0), (False, m, X, Y, 0, 256, 1)]:
        with pytest.raises(RuntimeError, match="invalid"):
            rb.matmul_quant_batch([bad])


@pytest.mark.parametrize("q6", [False, True])
def test_matmul_many_tiles(rb, oracle_lib, q6):
    """Several 32-token chunks and 256-row groups, ragged at both ends, and a repeat that must
    give the same bits."""
    rows, cols, T = 1000, 8192, 70
    m = synth.quant_matrix(900 + int(q6), rows, cols, q6)
    X = np.random.default_rng(17).standard_normal((T, cols)).astype(np.float32)
    dm, dX = dev(m), dev(X)
    Y = torch.zeros(T, rows, device="cuda")
    rb.matmul_quant_batch([(q6, dm, dX, Y, rows, cols, T)])
    first = Y.clone()
    rb.matmul_quant_batch([(q6, dm, dX, Y, rows, cols, T)])
    assert torch.equal(first, Y)
    assert O.maxrel(host(Y), _ref(q6, m, X, rows, cols)) < TOL


@pytest.mark.parametrize("q6", [False, True])
def test_matmul_activation_range(rb, oracle_lib, q6):
    """Each token is scaled on its own: magnitudes from 1e-4 to 1e4 side by side, a zero token,
    and a token of equal positive values (its sub-block sums are 32x its largest entry)."""
    rows, cols, T = 96, 4096, 12
    m = synth.quant_matrix(31 + int(q6), rows, cols, q6)
    rng = np.random.default_rng(3)
    X = rng.standard_normal((T, cols)).astype(np.float32)
    X *= (10.0 ** np.linspace(-4, 4, T)).astype(np.float32)[:, None]
    X[5] = 0
    X[7] = 3.0e4
    Y = torch.zeros(T, rows, device="cuda")
    rb.matmul_quant_batch([(q6, dev(m), dev(X), Y, rows, cols, T)])
    ref = _ref(q6, m, X, rows, cols)
    got = host(Y)
    for t in range(T):
        assert O.maxrel(got[t], ref[t]) < TOL, t


@pytest.mark.parametrize("q6", [False, True])
@pytest.mark.parametrize("cols", [32768, 33024])
def test_matmul_wide_rows(rb, oracle_lib, q6, cols):
    """128 blocks a row is the widest the staged kernel takes; 129 goes token by token."""
    rows, T = 40, 9
    m = synth.quant_matrix(cols + int(q6), rows, cols, q6)
    X = np.random.default_rng(cols).uniform(-1, 1, (T, cols)).astype(np.float32)
    Y = torch.zeros(T, rows, device="cuda")
    rb.matmul_quant_batch([(q6, dev(m), dev(X), Y, rows, cols, T)])
    assert O.maxrel(host(Y), _ref(q6, m, X, rows, cols)) < TOL


def test_matmul_mixed_batch(rb, oracle_lib):
    """One call mixing staged jobs of different widths (block counts that do not divide evenly
    into the split parts) with jobs that go token by token (T < 8, a Q6_K row that is not a
    multiple of 16 bytes)."""
    specs = [(False, 300, 2816, 20), (True, 100, 6144, 33), (False, 64, 512, 8), (True, 50, 512, 10),
             (False, 70, 2048, 3)]
    keep, jobs, refs = [], [], []
    for i, (q6, rows, cols, T) in enumerate(specs):
        m = synth.quant_matrix(700 + i, rows, cols, q6)
        X = np.random.default_rng(i).standard_normal((T, cols)).astype(np.float32)
        dm, dX, Y = dev(m), dev(X), torch.zeros(T, rows, device="cuda")
        keep.append((dm, dX, Y))
        jobs.append((q6, dm, dX, Y, rows, cols, T))
        refs.append(_ref(q6, m, X, rows, cols))
    rb.matmul_quant_batch(jobs)
    for (_, _, Y), ref in zip(keep, refs):
        assert O.maxrel(host(Y), ref) < TOL


@pytest.mark.parametrize("q6,rows,cols", [(False, 8192, 2048), (True, 2048, 4096)])
def test_matmul_prefill_chunk(rb, oracle_lib, q6, rows, cols):
    """One 256-token prefill chunk (the reference's MM_MAX_T) through a full-size projection of
    the stack (q+gate Q4_K; o / ssm_out Q6_K): every tile full, no split."""
    T = 256
    m = synth.quant_matrix(rows + int(q6), rows, cols, q6)
    X = np.random.default_rng(256).standard_normal((T, cols)).astype(np.float32)
    Y = torch.zeros(T, rows, device="cuda")
    rb.matmul_quant_batch([(q6, dev(m), dev(X), Y, rows, cols, T)])
    assert O.maxrel(host(Y), _ref(q6, m, X, rows, cols)) < TOL


@pytest.mark.parametrize("q6,rows,cols,T", [(False, 1000, 4096, 513), (True, 2000, 2048, 600), (False, 8200, 512, 64)])
def test_matmul_tensor_core_path(rb, oracle_lib, q6, rows, cols, T):
    """Shapes for the tcgen05 kernel (64 or more tokens, at least 64 tiles of 128 rows x 64
    tokens), ragged in rows and tokens, and a repeat that must give the same bits."""
    m = synth.quant_matrix(rows + T + int(q6), rows, cols, q6)
    X = np.random.default_rng(T).standard_normal((T, cols)).astype(np.float32)
    dm, dX = dev(m), dev(X)
    Y = torch.zeros(T, rows, device="cuda")
    rb.matmul_quant_batch([(q6, dm, dX, Y, rows, cols, T)])
    first = Y.clone()
    rb.matmul_quant_batch([(q6, dm, dX, Y, rows, cols, T)])
    assert torch.equal(first, Y)
    assert O.maxrel(host(Y), _ref(q6, m, X, rows, cols)) < TOL


@pytest.mark.parametrize("layer", ["deltanet", "attention"])
def test_matmul_layer_for_a_round_of_slots(rb, oracle_lib, layer):
    """One layer's projections for 64 tokens (a round of 64 slots through the step group): the
    call has fewer tcgen05 tiles than SMs, so the jobs with the most blocks are split along
    their blocks into parts whose partial planes are summed in part order (both layers: the
    2048 x 4096 Q6_K job in 2 parts, so that every CTA fits one wave). Same bits on a repeat."""
    T = 64
    shapes = ([(False, 8192, 2048), (False, 4096, 2048), (False, 32, 2048), (False, 32, 2048), (True, 2048, 4096)]
              if layer == "deltanet" else
              [(False, 8192, 2048), (False, 512, 2048), (True, 512, 2048), (True, 2048, 4096)])
    rng = np.random.default_rng(3)
    Xs = {c: rng.standard_normal((T, c)).astype(np.float32) for c in (2048, 4096)}
    dXs = {c: dev(x) for c, x in Xs.items()}
    keep, jobs, refs = [], [], []
    for i, (q6, rows, cols) in enumerate(shapes):
        m = synth.quant_matrix(200 + i, rows, cols, q6)
        dm, Y = dev(m), torch.zeros(T, rows, device="cuda")
        keep.append((dm, Y))
        jobs.append((q6, dm, dXs[cols], Y, rows, cols, T))
        refs.append(_ref(q6, m, Xs[cols], rows, cols))
    rb.matmul_quant_batch(jobs)
    first = [Y.clone() for _, Y in keep]
    rb.matmul_quant_batch(jobs)
    for (_, Y), f, ref in zip(keep, first, refs):
        assert torch.equal(f, Y)
        assert O.maxrel(host(Y), ref) < TOL


def test_matmul_mixed_sizes_one_call(rb, oracle_lib):
    """One call with jobs of very different sizes sharing one X (4096, 200 and 3 rows; both
    formats): the call's tiles are enough for the tcgen05 kernel, which takes all three, the
    smallest filling one partial tile."""
    T, cols = 300, 2048
    X = np.random.default_rng(77).standard_normal((T, cols)).astype(np.float32)
    dX = dev(X)
    specs = [(False, 4096), (True, 200), (False, 3)]   # 32 x 5, 2 x 5 and 1 x 5 tiles
    keep, jobs, refs = [], [], []
    for i, (q6, rows) in enumerate(specs):
        m = synth.quant_matrix(90 + i, rows, cols, q6)
        dm, Y = dev(m), torch.zeros(T, rows, device="cuda")
        keep.append((dm, Y))
        jobs.append((q6, dm, dX, Y, rows, cols, T))
        refs.append(_ref(q6, m, X, rows, cols))
    rb.matmul_quant_batch(jobs)
    for (_, Y), ref in zip(keep, refs):
        assert O.maxrel(host(Y), ref) < TOL
