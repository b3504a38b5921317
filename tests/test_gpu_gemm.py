"""Batched Q8_0 projections on the tensor cores (tcgen05, f16 operands, f32
accumulation) against the reference's CPU Q8_0 x f32 path
(qwen3_q8_0_matvec_range, qwen3.uya:1200-1231), one sequence at a time.

The f16 rounding of the dequantised weights and of the activations gives a
per-row error of about 2^-12 of the row's magnitude, so max |diff| over
||y||_2 stays near 1e-5; the test holds it to GEMM_TOL, ten times below the
north star's 1e-3."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import rel_row_err

pytestmark = pytest.mark.gpu

Q8_0 = 6
GEMM_TOL = 1e-4


def q80_tensor(name, rows, cols, seed):
    from minicpmo_b200 import gguf
    from minicpmo_b200.gpu import Tensor

    w = torch.randn((rows, cols), generator=torch.Generator().manual_seed(seed)) * 0.02
    return Tensor(name, gguf.quantize(w, Q8_0).numpy(), Q8_0, rows, cols)


@pytest.mark.parametrize(
    "rows,cols,n",
    [(1024, 4096, 1), (1024, 4096, 7), (1024, 4096, 16), (1024, 4096, 17), (1024, 4096, 32),
     (4096, 12288, 8), (384, 1024, 3), (6144, 4096, 32)],
)
def test_batched_q8_0_vs_reference_cpu(pkg, gpu_ctx, O, rows, cols, n):
    t = q80_tensor(f"bq80_{rows}_{cols}", rows, cols, seed=rows + cols)
    gpu_ctx.upload_tensor(t)
    x = np.random.Generator(np.random.PCG64(rows * 7 + n)).standard_normal((n, cols)).astype(np.float32)
    y = gpu_ctx.matmul_q8_0_batch(t, x)
    assert y.shape == (n, rows) and np.isfinite(y).all()
    for i in range(n):
        ref = O.matvec_f32(Q8_0, t.data, rows, cols, x[i])
        assert rel_row_err(y[i], ref) < GEMM_TOL, (i, rel_row_err(y[i], ref))
    # deterministic: split-K partials are added in a fixed order
    assert np.array_equal(gpu_ctx.matmul_q8_0_batch(t, x), y)


def test_batched_q8_0_rejects_bad_shapes(pkg, gpu_ctx):
    from minicpmo_b200.gpu import GpuError

    t = q80_tensor("bq80_bad", 128, 256, seed=1)
    gpu_ctx.upload_tensor(t)
    with pytest.raises(GpuError):
        gpu_ctx.matmul_q8_0_batch(t, np.zeros((33, 256), np.float32))
