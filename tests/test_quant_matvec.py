"""k-quant projections (kernel_cuda_matvec_quant_batch) against the reference's own CPU matvec
(matvec_q4_cpu / matvec_q6_cpu, kernels.c:405-431, 553-578, compiled into oracle/_ref; the oracle
restatement where it is absent). Tolerance 1e-5 maxrel: fp32 dot products over up to 4096 weights,
summed in a different order (the staged kernel sums on the tensor cores with the activation split
into two f16 halves, about 22 bits)."""
import numpy as np
import pytest
import torch

import oracle as O
from roaster_b200 import synth
from tests.gpu_util import dev, host

pytestmark = pytest.mark.gpu
TOL = 1e-5


def _ref(q6, m, x, rows, cols):
    return O.matvec_q(q6, m, x, rows, cols, impl="ref" if O.have_ref() else "port")


@pytest.mark.parametrize("q6", [False, True])
@pytest.mark.parametrize("rows,cols", [(1, 256), (64, 256), (300, 2048), (8192, 2048), (2048, 4096), (33, 4096),
                                       (40, 8192)])
def test_matvec(rb, oracle_lib, q6, rows, cols):
    """Shapes on both kernels: staged (16-byte rows up to 4096 weights) and the row kernel (Q6_K
    rows of 1 block, 8192 weights)."""
    m = synth.quant_matrix(rows + cols, rows, cols, q6)
    x = np.random.default_rng(rows).standard_normal(cols).astype(np.float32)
    dm, dx = dev(m), dev(x)
    y = torch.zeros(rows, device="cuda")
    rb.matvec_quant_batch([(q6, dm, dx, y, rows, cols)])
    assert O.maxrel(host(y), _ref(q6, m, x, rows, cols)) < TOL


@pytest.mark.parametrize("scale", [1e-6, 1.0, 3e4])
def test_activation_range(rb, oracle_lib, scale):
    """The power-of-two activation scaling keeps tiny and large vectors exact to the tolerance."""
    rows, cols = 96, 2048
    for q6 in (False, True):
        m = synth.quant_matrix(7, rows, cols, q6)
        x = (np.random.default_rng(8).standard_normal(cols) * scale).astype(np.float32)
        y = torch.zeros(rows, device="cuda")
        rb.matvec_quant_batch([(q6, dev(m), dev(x), y, rows, cols)])
        assert O.maxrel(host(y), _ref(q6, m, x, rows, cols)) < TOL


def test_unaligned_matrix_uses_row_kernel(rb, oracle_lib):
    """A Q6_K matrix on a 2-byte (not 16-byte) boundary takes the row kernel, same results."""
    rows, cols = 48, 2048
    m = synth.quant_matrix(9, rows, cols, True)
    buf = torch.zeros(m.size + 16, dtype=torch.uint8, device="cuda")
    buf[2:2 + m.size] = dev(m)
    x = np.random.default_rng(10).standard_normal(cols).astype(np.float32)
    y = torch.zeros(rows, device="cuda")
    rb.matvec_quant_batch([(True, buf.data_ptr() + 2, dev(x), y, rows, cols)])
    assert O.maxrel(host(y), _ref(True, m, x, rows, cols)) < TOL


def test_mixed_batch(rb, oracle_lib):
    """One call: Q4_K and Q6_K jobs of a layer's projection shapes, each with its own vector."""
    shapes = [(False, 8192, 2048), (False, 512, 2048), (True, 512, 2048), (True, 2048, 4096), (False, 32, 2048),
              (False, 2048, 512), (True, 5, 256)]
    keep, jobs, refs = [], [], []
    for i, (q6, r, c) in enumerate(shapes):
        m = synth.quant_matrix(100 + i, r, c, q6)
        x = np.random.default_rng(200 + i).standard_normal(c).astype(np.float32)
        dm, dx, y = dev(m), dev(x), torch.zeros(r, device="cuda")
        keep.append((dm, dx, y))
        jobs.append((q6, dm, dx, y, r, c))
        refs.append(_ref(q6, m, x, r, c))
    rb.matvec_quant_batch(jobs)
    for (dm, dx, y), ref in zip(keep, refs):
        assert O.maxrel(host(y), ref) < TOL


def test_many_jobs(rb, oracle_lib):
    """More jobs than one launch carries (64): the call splits them."""
    keep, jobs, refs = [], [], []
    for i in range(70):
        q6, r, c = bool(i % 3 == 0), 16 + 8 * (i % 5), 256 * (1 + i % 4)
        m = synth.quant_matrix(300 + i, r, c, q6)
        x = np.random.default_rng(400 + i).standard_normal(c).astype(np.float32)
        dm, dx, y = dev(m), dev(x), torch.zeros(r, device="cuda")
        keep.append((dm, dx, y))
        jobs.append((q6, dm, dx, y, r, c))
        refs.append(_ref(q6, m, x, r, c))
    rb.matvec_quant_batch(jobs)
    for (dm, dx, y), ref in zip(keep, refs):
        assert O.maxrel(host(y), ref) < TOL


@pytest.mark.parametrize("q6", [False, True])
def test_whole_tiles_and_repeat(rb, oracle_lib, q6):
    """A call with more tiles (16 rows) than twice the warps keeps tiles whole (y stored directly);
    small calls split tiles into parts whose partials meet in a per-tile counter that returns to
    zero, so calling again gives the same result."""
    rows, cols = 80000, 256
    m = synth.quant_matrix(31, rows, cols, q6)
    x = np.random.default_rng(32).standard_normal(cols).astype(np.float32)
    ref = _ref(q6, m, x, rows, cols)
    dm, dx = dev(m), dev(x)
    for _ in range(2):
        y = torch.zeros(rows, device="cuda")
        rb.matvec_quant_batch([(q6, dm, dx, y, rows, cols)])
        assert O.maxrel(host(y), ref) < TOL
    m2 = synth.quant_matrix(33, 64, 4096, q6)
    x2 = np.random.default_rng(34).standard_normal(4096).astype(np.float32)
    ref2 = _ref(q6, m2, x2, 64, 4096)
    dm2, dx2 = dev(m2), dev(x2)
    outs = []
    for _ in range(3):
        y2 = torch.zeros(64, device="cuda")
        rb.matvec_quant_batch([(q6, dm2, dx2, y2, 64, 4096)])
        outs.append(host(y2))
        assert O.maxrel(outs[-1], ref2) < TOL
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])   # fixed summation order


def test_rejects_ragged_cols(rb):
    m = torch.zeros(144, dtype=torch.uint8, device="cuda")
    x = torch.zeros(300, device="cuda")
    y = torch.zeros(1, device="cuda")
    with pytest.raises(RuntimeError, match="multiple of 256"):
        rb.matvec_quant_batch([(False, m, x, y, 1, 300)])
