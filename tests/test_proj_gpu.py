"""b2a_proj (decode-batch projection with the norm / residual add / SwiGLU fused) on the GPU.

The reference is the same arithmetic in float64 with the kernel's roundings
placed where the kernel places them (the norm's operand x * w_n rounded to
bf16, the per-row scale on the product, gate and up and silu(gate) rounded as
the unfused 16-bit form rounds them; python/minisgl_mlx/models/transformer.py
:26-30, :41-42, :64-69, :80-82). What is left between the two is the fp32
accumulation order of the tensor cores, so every stored value is within one
bf16 step of the reference (four after the SwiGLU's chained roundings: a flip
of gate's or up's rounding moves the product by up to 2^-7 each) plus a
floor of 1e-5 of the output scale for values that cancel to almost nothing
(there the fp32 sum's own error is larger than a bf16 step of the value), and
close to the unrounded float64 product too.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

# (N, K, mode): Qwen3-0.6B's qkv (RMSNorm in front), o (+ residual), gate_up (RMSNorm + SwiGLU),
# down (+ residual), and the test model's shapes
SHAPES = [(4096, 1024, 0, True), (1024, 2048, 1, False), (6144, 1024, 2, True), (1024, 3072, 1, False),
          (4096, 256, 0, True), (256, 2048, 1, False), (1024, 256, 2, True), (256, 512, 1, False)]
ROWS = [1, 3, 8, 9, 16, 17, 32, 33, 50, 64]


def _bf16(t):
    import torch

    return t.to(torch.bfloat16).to(torch.float64)


def _ulp(y):
    import torch

    a = y.abs().clamp_min(1e-30)
    return torch.exp2(torch.floor(torch.log2(a)) - 7)


def _within(got, want, steps):
    """max over elements of |got - want| / (steps bf16 steps of want + 1e-5 of the scale)."""
    floor = 1e-5 * want.abs().max()
    r = (got - want).abs() / (steps * _ulp(want) + floor)
    i = int(r.argmax())
    if r.flatten()[i] > 1.0:  # say where, for the failure message
        print("worst element", divmod(i, want.shape[1]), "got", got.flatten()[i].item(), "want",
              want.flatten()[i].item(), "scale", want.abs().max().item())
    return r.max().item()


def _reference(x, w, mode, norm_w, eps, res):
    """float64 with the kernel's rounding points; returns (mirrored, unrounded)."""
    import torch

    xd, wd = x.double(), w.double()
    if norm_w is not None:
        inv = torch.rsqrt((xd * xd).mean(dim=1, keepdim=True) + eps)
        acc = _bf16(xd * norm_w.double()) @ wd.T * inv
        exact = (xd * inv * norm_w.double()) @ wd.T
    else:
        acc = xd @ wd.T
        exact = acc
    if mode == 0:
        return _bf16(acc), exact
    if mode == 1:
        return _bf16(res.double() + acc), res.double() + exact
    F = w.shape[0] // 2
    g, u = _bf16(acc[:, :F]), _bf16(acc[:, F:])
    s = _bf16(g / (1 + torch.exp(-g)))
    ge, ue = exact[:, :F], exact[:, F:]
    return _bf16(s * u), ge / (1 + torch.exp(-ge)) * ue


@pytest.mark.parametrize("M", ROWS)
@pytest.mark.parametrize("N,K,mode,norm", SHAPES)
def test_proj_matches_float64(N, K, mode, norm, M):
    import torch

    from minisgl_b200.engine.model import proj

    gen = torch.Generator(device="cuda").manual_seed(1000 * M + N + K + mode)
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn((N, K), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    norm_w = (1 + 0.1 * torch.randn(K, device="cuda", generator=gen)).to(torch.bfloat16) if norm else None
    res = torch.randn((M, N), device="cuda", generator=gen).to(torch.bfloat16) if mode == 1 else None
    want, exact = _reference(x, w, mode, norm_w, 1e-6, res)
    got = proj(x, w, mode, norm_w, 1e-6, res=res).double()
    torch.cuda.synchronize()
    r = _within(got, want, 4.0 if mode == 2 else 1.0)
    assert r <= 1.0, r
    scale = exact.abs().max().item()
    assert (got - exact).abs().max().item() <= 2e-2 * scale


def test_proj_residual_in_place_and_strided_rows():
    """out = res (the hidden rows updated in place) and row strides wider than the rows."""
    import torch

    from minisgl_b200.engine.model import PROJ_RESIDUAL, proj

    gen = torch.Generator(device="cuda").manual_seed(7)
    M, N, K = 20, 1024, 2048
    xbig = torch.randn((M, K + 64), device="cuda", generator=gen).to(torch.bfloat16)
    x = xbig[:, 8: 8 + K]  # row stride K + 64, 16-byte aligned start
    w = (torch.randn((N, K), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    h = torch.randn((M, N), device="cuda", generator=gen).to(torch.bfloat16)
    want, _ = _reference(x, w, 1, None, 0.0, h.clone())
    proj(x, w, PROJ_RESIDUAL, res=h, out=h)
    torch.cuda.synchronize()
    assert _within(h.double(), want, 1.0) <= 1.0


def test_proj_inside_cuda_graph():
    """Captured and replayed (the engine's decode graphs), with new inputs copied in."""
    import torch

    from minisgl_b200.engine.model import PROJ_SWIGLU, proj

    gen = torch.Generator(device="cuda").manual_seed(3)
    M, N, K = 32, 6144, 1024
    x = torch.randn((M, K), device="cuda", generator=gen).to(torch.bfloat16)
    w = (torch.randn((N, K), device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    nw = torch.ones(K, device="cuda", dtype=torch.bfloat16)
    proj(x, w, PROJ_SWIGLU, nw, 1e-6)  # first call outside capture (launch shape, shared memory)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
        out = proj(x, w, PROJ_SWIGLU, nw, 1e-6)
    torch.cuda.current_stream().wait_stream(s)
    for seed in (11, 12):
        x.copy_(torch.randn((M, K), device="cuda", generator=gen.manual_seed(seed)).to(torch.bfloat16))
        g.replay()
        torch.cuda.synchronize()
        want, _ = _reference(x, w, 2, nw, 1e-6, None)
        assert _within(out.double(), want, 4.0) <= 1.0


def test_proj_rejects_unsupported_shapes():
    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.engine.model import proj

    x = torch.zeros((65, 1024), device="cuda", dtype=torch.bfloat16)
    w = torch.zeros((1024, 1024), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(nat.B200AttnError, match="at most 64"):
        proj(x, w, 0)
    with pytest.raises(nat.B200AttnError, match="multiple of 128"):
        proj(x[:4, :1000], w[:, :1000].contiguous(), 0)
    with pytest.raises(nat.B200AttnError, match="bf16 only"):
        proj(x[:4].float(), w.float(), 0)


def test_engine_bf16_fused_projections_match_unfused():
    """The bf16 model's decode-step logits with the fused b2a_proj layers against the
    unfused cuBLAS + b2a_rmsnorm + b2a_swiglu layers on the same state."""
    import torch

    from minisgl_b200.core import SamplingParams
    from minisgl_b200.engine import LLM, EngineConfig, qwen3_0_6b_spec

    rng = np.random.default_rng(9)
    prompts = [rng.integers(0, 10000, int(rng.integers(50, 200))).astype(np.int32) for _ in range(12)]
    outs = {}
    for fused in (True, False):
        cfg = EngineConfig(spec=qwen3_0_6b_spec(), dtype="bfloat16", max_running_req=16, page_size=16,
                           num_tokens=8192, max_extend_tokens=4096, cuda_graph_max_bs=16, fused_proj=fused)
        llm = LLM(cfg)
        assert llm.engine.model.fused_proj == fused
        res = llm.generate(prompts, [SamplingParams(max_tokens=6, ignore_eos=True) for _ in prompts])
        outs[fused] = [o["token_ids"] for o in res]
        llm.engine.shutdown()
        del llm
        torch.cuda.empty_cache()
    # random-init weights give near-flat logits, so a greedy token can flip on a rounding
    # difference; the first decode token after an identical prefill must mostly agree
    same = sum(a[:2] == b[:2] for a, b in zip(outs[True], outs[False]))
    assert same >= len(prompts) - 2, (outs[True], outs[False])
