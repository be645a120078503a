"""FP16 / BF16 input-output softmax and RMSNorm (opl_*_f16 / *_bf16) against
the CPU oracle run on the same inputs upcast to FP32: the kernels compute in
FP32 and round once, so every output is within one unit in the last place of
the storage type of the oracle's value (fp16: 2^-10 relative, bf16: 2^-7)."""
from __future__ import annotations

import numpy as np
import pytest

import operatorlib
from oracle import oracle as orc

pytestmark = pytest.mark.gpu

CASES = [(4096, 1024), (4097, 1023), (19, 128), (5, 4104), (3, 8192), (2, 16384),
         (2, 40000), (1, 1), (7, 13)]


def _torch_dtype(name):
    import torch

    return {"f16": torch.float16, "bf16": torch.bfloat16}[name]


def _ulp_check(got, want, name):
    rel = 2.0 ** -10 if name == "f16" else 2.0 ** -7
    tiny = 6e-8 if name == "f16" else 1e-38
    assert np.all(np.abs(got - want) <= rel * np.abs(want) + tiny), \
        np.max(np.abs(got - want) / (np.abs(want) + tiny))


@pytest.mark.parametrize("name", ["f16", "bf16"])
@pytest.mark.parametrize("rows,cols", CASES)
def test_softmax16(cuda, stream, name, rows, cols):
    import torch

    dt = _torch_dtype(name)
    x = torch.from_numpy(np.random.default_rng(rows + cols).normal(0, 2, (rows, cols))
                         .astype(np.float32)).to(cuda).to(dt)
    y = torch.empty_like(x)
    operatorlib.softmax_into(x, y)
    stream.synchronize()
    want = orc.softmax(x.float().cpu().numpy())
    _ulp_check(y.float().cpu().numpy(), want, name)


@pytest.mark.parametrize("name", ["f16", "bf16"])
@pytest.mark.parametrize("rows,cols", CASES)
def test_rmsnorm16(cuda, stream, name, rows, cols):
    import torch

    dt = _torch_dtype(name)
    rng = np.random.default_rng(rows * 3 + cols)
    x = torch.from_numpy(rng.normal(0, 1, (rows, cols)).astype(np.float32)).to(cuda).to(dt)
    w = torch.from_numpy(rng.normal(1, 0.1, cols).astype(np.float32)).to(cuda).to(dt)
    y = torch.empty_like(x)
    operatorlib.rmsnorm_into(x, w, y, 1e-6)
    stream.synchronize()
    want = orc.rmsnorm(x.float().cpu().numpy(), w.float().cpu().numpy(), 1e-6)
    _ulp_check(y.float().cpu().numpy(), want, name)


def test_row16_rejects_bad_arguments():
    lib = operatorlib.capi()
    assert lib.opl_softmax_f16(None, 0x1000, 2, 2, None) == 1
    assert lib.opl_rmsnorm_bf16(0x1000, 0x1000, 0x1000, 2, 2, 0.0, None) == 1
