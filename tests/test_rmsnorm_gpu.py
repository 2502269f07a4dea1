"""b2a_rmsnorm (the engine harness's RMSNorm, reference models/transformer.py:77-82 and the
last-token gather + final norm of :109-113) against a plain PyTorch fp32 reference."""

from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu


def _ref(x, w, eps, rows=None):
    import torch

    xf = x.float() if rows is None else x.float()[rows.long()]
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float())


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
@pytest.mark.parametrize("T,H", [(1, 1024), (128, 1024), (37, 256), (300, 2048), (64, 4096)])
@pytest.mark.parametrize("gather", [False, True])
def test_rmsnorm_matches_fp32_reference(dtype, T, H, gather):
    import torch

    if dtype == "float32" and H > 2048:
        pytest.skip("fp32 rows hold at most 16 vectors of 4 per lane (H <= 2048)")

    from minisgl_b200.engine.model import rms_norm

    dt = getattr(torch, dtype)
    g = torch.Generator(device="cuda").manual_seed(T * 13 + H)
    x = (torch.randn((T, H), generator=g, device="cuda") * 3).to(dt)
    w = (torch.rand((H,), generator=g, device="cuda") + 0.5).to(dt)
    rows = None
    if gather:
        rows = torch.randint(0, T, (max(1, T // 3),), generator=g, device="cuda", dtype=torch.int32)
    y = rms_norm(x, w, 1e-6, rows)
    torch.cuda.synchronize()
    ref = _ref(x, w, 1e-6, rows)
    # one rounding to the storage type: within one ulp of the fp32 result
    tol = {"float32": 1e-5, "bfloat16": 2 ** -7, "float16": 2 ** -10}[dtype]
    err = ((y.float() - ref).abs() / ref.abs().clamp_min(1e-3)).max().item()
    assert err <= tol, err


def test_rmsnorm_strided_rows_and_bad_gather_index():
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.engine.model import rms_norm

    g = torch.Generator(device="cuda").manual_seed(5)
    buf = torch.randn((16, 1024 + 64), generator=g, device="cuda").to(torch.bfloat16)
    x = buf[:, :1024]  # row stride 1088 elements
    w = torch.ones(1024, dtype=torch.bfloat16, device="cuda")
    y = rms_norm(x, w, 1e-6)
    assert torch.allclose(y.float(), _ref(x, w, 1e-6), rtol=2 ** -7, atol=0)
    rows = torch.tensor([3, 99, 15], dtype=torch.int32, device="cuda")  # 99 is outside the 16 rows
    y = rms_norm(x, w, 1e-6, rows)
    code = ctypes.c_int(-1)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert code.value == 32
    ok = torch.tensor([0, 2])
    assert torch.allclose(y[ok].float(), _ref(x, w, 1e-6, rows[ok]), rtol=2 ** -7, atol=0)


def test_rmsnorm_rejects_rows_wider_than_compiled():
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.engine.model import rms_norm

    x = torch.zeros((2, 4096), dtype=torch.float32, device="cuda")
    with pytest.raises(nat.B200AttnError, match="not compiled"):
        rms_norm(x, torch.ones(4096, device="cuda"), 1e-6)
