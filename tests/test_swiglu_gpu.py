"""b2a_swiglu (the engine harness's SwiGLU, reference models/transformer.py:26-30)
against torch's unfused ``F.silu(gate) * up`` on the same tensors."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def _swiglu_call(gu, row_stride, rows, F, out):
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.kvcache.pool import dtype_code

    nat.call("b2a_swiglu", gu.data_ptr(), row_stride, out.data_ptr(), rows, F, dtype_code(gu.dtype),
             torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("rows,F,pad", [(1, 2, 0), (7, 3072, 0), (128, 3072, 0), (33, 1000, 24)])
def test_swiglu_matches_unfused_torch(dtype, rows, F, pad):
    import torch
    import torch.nn.functional as Fn

    dt = getattr(torch, dtype)
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + F)
    # pad > 0: gate/up rows are a slice of a wider buffer (row stride 2F + pad)
    buf = (torch.randn((rows, 2 * F + pad), generator=g, device="cuda") * 4).to(dt)
    gu = buf[:, : 2 * F]
    gate, up = gu[:, :F], gu[:, F:]
    ref = Fn.silu(gate) * up
    out = torch.empty((rows, F), dtype=dt, device="cuda")
    _swiglu_call(gu, buf.stride(0), rows, F, out)
    torch.cuda.synchronize()
    err = (out.float() - ref.float()).abs()
    # same roundings as the unfused form: equal up to one unit in the last place
    ulp = {"float32": 2.0 ** -23, "bfloat16": 2.0 ** -7, "float16": 2.0 ** -10}[dtype]
    bound = ref.float().abs() * ulp + 1e-30
    assert bool((err <= bound).all()), float((err / bound).max())


def test_swiglu_rejects_bad_sizes():
    import torch

    x = torch.zeros((4, 8), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((4, 4), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="even"):
        _swiglu_call(x, 8, 4, 3, out)
    with pytest.raises(ValueError, match="row_stride"):
        _swiglu_call(x, 6, 4, 4, out)
    _swiglu_call(x, 8, 0, 4, out)  # nothing to do
