"""The C-ABI library: it loads without a GPU, exports every function include/roaster_cuda.h
declares, and fails cleanly (returns -1 with a message) when no B200 is usable. CPU only."""
import ctypes as C
import os
import subprocess

import pytest

import roaster_b200 as R


def test_library_exports_every_declared_symbol():
    lib = R.lib()
    declared = R.header_symbols()
    assert len(declared) >= 15
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", R.LIB_PATH], capture_output=True, text=True)
    exported = {ln.split()[-1] for ln in out.stdout.splitlines() if " T " in ln}
    assert set(declared) <= exported


def test_header_compiles_as_c(tmp_path):
    src = tmp_path / "t.c"
    src.write_text('#include "roaster_cuda.h"\nint main(void){ KernelAttnDecodeJob j; '
                   'KernelDeltaStepJob d; KernelDeltaPrefillJob e; KernelDeltaPreopJob f; KernelDeltaPostopJob g; (void)j; (void)d; (void)e; (void)f; (void)g; return 0; }\n')
    inc = os.path.join(os.path.dirname(R.LIB_PATH), "..", "include")
    out = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", inc, str(src), "-o",
                          str(tmp_path / "t")], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr


def test_struct_layouts_match_c(tmp_path):
    """ctypes mirrors have the C sizes and offsets."""
    src = tmp_path / "s.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "roaster_cuda.h"\n'
                   'int main(void){ printf("%zu %zu %zu %zu %zu %zu %zu %zu\\n", '
                   'sizeof(KernelAttnDecodeJob), offsetof(KernelAttnDecodeJob, append), '
                   'sizeof(KernelDeltaStepJob), offsetof(KernelAttnDecodeJob, out), '
                   'sizeof(KernelAttnPrefillJob), offsetof(KernelAttnPrefillJob, dtype), '
                   'sizeof(KernelDeltaPrefillJob), offsetof(KernelDeltaPrefillJob, T)); '
                   'printf("%zu %zu %zu %zu\\n", sizeof(KernelDeltaPreopJob), offsetof(KernelDeltaPreopJob, T), '
                   'sizeof(KernelDeltaPostopJob), offsetof(KernelDeltaPostopJob, T)); '
                   'printf("%zu %zu %zu %zu\\n", sizeof(KernelCudaMatvecJob), offsetof(KernelCudaMatvecJob, cols), '
                   'sizeof(KernelCudaMatmulJob), offsetof(KernelCudaMatmulJob, T)); '
                   'return 0; }\n')
    inc = os.path.join(os.path.dirname(R.LIB_PATH), "..", "include")
    exe = tmp_path / "s"
    subprocess.run(["gcc", "-I", inc, str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    assert vals == [C.sizeof(R.KernelAttnDecodeJob), R.KernelAttnDecodeJob.append.offset,
                    C.sizeof(R.KernelDeltaStepJob), R.KernelAttnDecodeJob.out.offset,
                    C.sizeof(R.KernelAttnPrefillJob), R.KernelAttnPrefillJob.dtype.offset,
                    C.sizeof(R.KernelDeltaPrefillJob), R.KernelDeltaPrefillJob.T.offset,
                    C.sizeof(R.KernelDeltaPreopJob), R.KernelDeltaPreopJob.T.offset,
                    C.sizeof(R.KernelDeltaPostopJob), R.KernelDeltaPostopJob.T.offset,
                    C.sizeof(R.KernelCudaMatvecJob), R.KernelCudaMatvecJob.cols.offset,
                    C.sizeof(R.KernelCudaMatmulJob), R.KernelCudaMatmulJob.T.offset]


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.mark.skipif(_has_gpu(), reason="checks the no-GPU failure path")
def test_no_gpu_fails_cleanly():
    lib = R.lib()
    assert lib.kernel_cuda_init(0) == -1
    assert R.last_error()
    jobs = (R.KernelDeltaStepJob * 1)()
    assert lib.kernel_deltanet_step_batch(jobs, 1) == -1
    assert lib.kernel_cuda_alloc(1024) is None
