"""GPU parity of the fused RoPE + KV store (reference layers.py:45-56,103-109; kvcache/pool.py:47-50).

* rotated q/k within tolerance of the oracle's rotation (same fp32 angle rule)
* pool rows at out_loc BIT-identical to the rotated k returned to the caller and to v
* every other pool row untouched
* strided q/k/v views (slices of one fused qkv buffer) are handled in place
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import TOL, max_abs, rand, to_dev, to_np, torch_dtype
from oracle import attention as O

pytestmark = pytest.mark.gpu


def _setup(T, Hq, Hkv, D, dtype, N, seed, max_pos=131072):
    rng = np.random.default_rng(seed)
    qkv = rand(rng, (T, (Hq + 2 * Hkv) * D), dtype)
    positions = rng.integers(0, max_pos, size=T).astype(np.int32)
    positions[:2] = [0, 1]
    out_loc = rng.permutation(N)[:T].astype(np.int32)
    return rng, qkv, positions, out_loc


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("rot", [128, 64])
def test_rope_store_strided_qkv(dtype, rot):
    import torch

    from minisgl_b200.config import RotaryConfig
    from minisgl_b200.kvcache import MHAKVCache
    from minisgl_b200.layers import RotaryEmbedding

    T, Hq, Hkv, D, N = 300, 16, 8, 128, 4096
    rng, qkv, positions, out_loc = _setup(T, Hq, Hkv, D, dtype, N, seed=1)
    kv = MHAKVCache(2, N, Hkv, D, torch_dtype(dtype))
    kv.k[1].copy_(torch.from_numpy(rand(rng, (N, Hkv, D), dtype)))
    kv.v[1].copy_(torch.from_numpy(rand(rng, (N, Hkv, D), dtype)))
    before_k = kv.k[1].clone()
    before_v = kv.v[1].clone()
    other_layer = kv.k[0].clone()

    buf = to_dev(qkv, dtype)
    q = buf[:, : Hq * D].view(T, Hq, D)
    k = buf[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = buf[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    rope = RotaryEmbedding(RotaryConfig(D, rot, 1e6, 131072))
    rope.rope_store_(q, k, v, torch.from_numpy(positions).cuda(), torch.from_numpy(out_loc).cuda(), kv, 1)
    torch.cuda.synchronize()

    hq = qkv[:, : Hq * D].reshape(T, Hq, D)
    hk = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    hv = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    ref_q = O.rope(hq, positions, rot, rope.inv_freq_host, 1.0, dtype)
    ref_k = O.rope(hk, positions, rot, rope.inv_freq_host, 1.0, dtype)
    tol = 2e-6 if dtype == "float32" else TOL["bfloat16"]
    assert max_abs(to_np(q), ref_q) <= tol * 4
    assert max_abs(to_np(k), ref_k) <= tol * 4
    if dtype == "bfloat16":
        # only rounding-boundary ties may land one bf16 ulp apart
        assert np.mean(to_np(k) == ref_k) > 0.99
    # v is untouched
    np.testing.assert_array_equal(to_np(v), hv)
    # slots: bit-exact
    loc = torch.from_numpy(out_loc).long().cuda()
    assert torch.equal(kv.k[1][loc].view(torch.int16 if dtype != "float32" else torch.int32),
                       k.contiguous().view(torch.int16 if dtype != "float32" else torch.int32))
    assert torch.equal(kv.v[1][loc], v.contiguous())
    mask = torch.ones(N, dtype=torch.bool, device="cuda")
    mask[loc] = False
    assert torch.equal(kv.k[1][mask], before_k[mask])
    assert torch.equal(kv.v[1][mask], before_v[mask])
    assert torch.equal(kv.k[0], other_layer)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16", "float16"])
def test_store_kv_bit_exact(dtype):
    import torch

    from minisgl_b200.kvcache import MHAKVCache

    rng = np.random.default_rng(2)
    T, Hkv, D, N = 77, 4, 64, 1000
    kv = MHAKVCache(3, N, Hkv, D, torch_dtype(dtype))
    k = to_dev(rand(rng, (T, Hkv, D), "float32"), dtype)
    v = to_dev(rand(rng, (T, Hkv, D), "float32"), dtype)
    loc = torch.from_numpy(rng.permutation(N)[:T].astype(np.int32)).cuda()
    kv.store_kv(k, v, loc, 2)
    torch.cuda.synchronize()
    assert torch.equal(kv.k[2][loc.long()], k) and torch.equal(kv.v[2][loc.long()], v)
    rest = torch.ones(N, dtype=torch.bool, device="cuda")
    rest[loc.long()] = False
    assert int(kv.k[2][rest].abs().sum()) == 0 and int(kv.v[2][rest].abs().sum()) == 0
    assert int(kv.k[0].abs().sum()) == 0


def test_rope_standalone_matches_oracle_large_positions():
    import torch

    from minisgl_b200.config import RotaryConfig
    from minisgl_b200.layers import RotaryEmbedding

    rng = np.random.default_rng(3)
    x = rand(rng, (513, 4, 128), "float32")
    pos = rng.integers(0, 131072, size=513).astype(np.int32)
    cfg = RotaryConfig(128, 128, 5e5, 131072, {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                               "high_freq_factor": 4.0,
                                               "original_max_position_embeddings": 8192})
    rope = RotaryEmbedding(cfg)
    y = rope(to_dev(x, "float32"), torch.from_numpy(pos).cuda())
    torch.cuda.synchronize()
    ref = O.rope(x, pos, 128, rope.inv_freq_host, rope.scale, "float32")
    assert max_abs(to_np(y), ref) <= 1e-5
    # linear scaling folds 1/factor into the position
    cfg = RotaryConfig(128, 128, 1e4, 8192, {"rope_type": "linear", "factor": 4.0})
    rope = RotaryEmbedding(cfg)
    y = rope(to_dev(x, "float32"), torch.from_numpy(pos).cuda())
    ref = O.rope(x, pos, 128, rope.inv_freq_host, 0.25, "float32")
    assert max_abs(to_np(y), ref) <= 1e-5


def _rms_rows(x: np.ndarray, w: np.ndarray, eps: float, dtype: str) -> np.ndarray:
    """models/transformer.py:54-56 (nn.RMSNorm over head_dim) in float64, rounded to dtype."""
    x = x.astype(np.float64)
    y = x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w.astype(np.float64)
    return O.round_to(y, dtype)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("q_out", [False, True])
def test_qknorm_rope_store(dtype, q_out):
    """q/k RMSNorm fused in front of RoPE + store: oracle = norm (rounded) then rope."""
    import torch

    from minisgl_b200.config import RotaryConfig
    from minisgl_b200.kvcache import MHAKVCache
    from minisgl_b200.layers import RotaryEmbedding

    T, Hq, Hkv, D, N, eps = 257, 16, 8, 128, 2048, 1e-6
    rng, qkv, positions, out_loc = _setup(T, Hq, Hkv, D, dtype, N, seed=3)
    qkv = O.round_to(qkv * 3.0, dtype)  # rows far from unit RMS
    wq = O.round_to(rng.uniform(0.5, 1.5, D).astype(np.float32), dtype)
    wk = O.round_to(rng.uniform(0.5, 1.5, D).astype(np.float32), dtype)
    kv = MHAKVCache(1, N, Hkv, D, torch_dtype(dtype))
    buf = to_dev(qkv, dtype)
    q = buf[:, : Hq * D].view(T, Hq, D)
    k = buf[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = buf[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    rope = RotaryEmbedding(RotaryConfig(D, D, 1e6, 131072))
    qo = torch.empty((T, Hq, D), dtype=torch_dtype(dtype), device="cuda") if q_out else None
    rope.rope_store_(q, k, v, torch.from_numpy(positions).cuda(), torch.from_numpy(out_loc).cuda(), kv, 0,
                     to_dev(wq, dtype), to_dev(wk, dtype), eps, q_out=qo)
    torch.cuda.synchronize()

    hq = qkv[:, : Hq * D].reshape(T, Hq, D)
    hk = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D)
    hv = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
    ref_q = O.rope(_rms_rows(hq, wq, eps, dtype), positions, D, rope.inv_freq_host, 1.0, dtype)
    ref_k = O.rope(_rms_rows(hk, wk, eps, dtype), positions, D, rope.inv_freq_host, 1.0, dtype)
    # the normalised rows reach |x| ~ 5, where one bf16 ulp is 2^-5: the bf16 bound scales
    # with the magnitude (2e-2 relative above 1, the absolute 2e-2 below)
    tol = 1e-5 if dtype == "float32" else TOL["bfloat16"]

    def rel_err(got, ref):
        return float(np.max(np.abs(got.astype(np.float64) - ref) / np.maximum(1.0, np.abs(ref))))

    got_q = to_np(qo if q_out else q)
    assert rel_err(got_q, ref_q) <= tol
    assert rel_err(to_np(k), ref_k) <= tol
    # the pool holds exactly the returned k and the untouched v
    assert np.array_equal(to_np(kv.k[0])[out_loc], to_np(k))
    assert np.array_equal(to_np(kv.v[0])[out_loc], hv)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("T,Hq,Hkv", [(3000, 16, 8), (37, 32, 8), (5, 4, 1)])
@pytest.mark.parametrize("norm", [False, True])
def test_token_path_matches_row_path(dtype, T, Hq, Hkv, norm):
    """The token-major fast path (16-bit, D = rot = 128, rows on 16 bytes) against the
    row-per-warp kernel, which a row stride that is not a multiple of 8 elements selects.
    Covers one warp per token (large T), several warps per token, and more q/k rows than
    one register pass holds (32q/8kv)."""
    import torch

    from minisgl_b200.config import RotaryConfig
    from minisgl_b200.kvcache import MHAKVCache
    from minisgl_b200.layers import RotaryEmbedding

    D, N, eps = 128, 4096, 1e-6
    rng, qkv, positions, out_loc = _setup(T, Hq, Hkv, D, dtype, max(N, T), seed=11)
    N = max(N, T)
    W = (Hq + 2 * Hkv) * D
    rope = RotaryEmbedding(RotaryConfig(D, D, 1e6, 131072))
    wq = to_dev(O.round_to(rng.uniform(0.5, 1.5, D).astype(np.float32), dtype), dtype) if norm else None
    wk = to_dev(O.round_to(rng.uniform(0.5, 1.5, D).astype(np.float32), dtype), dtype) if norm else None
    pos_d, loc_d = torch.from_numpy(positions).cuda(), torch.from_numpy(out_loc).cuda()
    outs = []
    for pad in (0, 1):  # pad 0: fast path; pad 1: odd row stride -> row kernel
        buf = torch.zeros((T, W + pad), dtype=torch_dtype(dtype), device="cuda")
        buf[:, :W] = to_dev(qkv, dtype)
        q = buf[:, : Hq * D].view(T, Hq, D) if pad == 0 else buf[:, : Hq * D].unflatten(1, (Hq, D))
        k = buf[:, Hq * D:(Hq + Hkv) * D].unflatten(1, (Hkv, D))
        v = buf[:, (Hq + Hkv) * D: W].unflatten(1, (Hkv, D))
        kv = MHAKVCache(1, N, Hkv, D, torch_dtype(dtype))
        rope.rope_store_(q, k, v, pos_d, loc_d, kv, 0, wq, wk, eps)
        torch.cuda.synchronize()
        outs.append((q.float().cpu(), k.float().cpu(), kv.k[0].float().cpu(), kv.v[0].float().cpu()))
    for a, b in zip(outs[0], outs[1]):
        if norm:
            # the RMSNorm's sum of squares is added in another order: a normalised element
            # may move by one ulp, which the rotation carries into outputs of the row's scale
            # (|x| <~ 4 here); almost every element stays bit-equal
            ulp = 2.0 ** -7 if dtype == "bfloat16" else 2.0 ** -10
            assert float((a - b).abs().max()) <= 2 * ulp * 4
            assert float((a == b).float().mean()) > 0.95
        else:
            assert torch.equal(a, b)
