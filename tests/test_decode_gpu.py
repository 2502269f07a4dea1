"""GPU parity of paged decode attention against the CPU oracle.

* test_paged_decode_kernel restates the reference's kernel test
  (tests/test_attention.py:19-39): the same head shapes, dtypes, N=4096, B=7,
  lens [1, 2, 17, 31, 32, 33, 700] on disjoint permuted slots, now against an
  fp64 oracle with the BASELINE tolerances (1e-5 fp32, 2e-2 bf16).
* the split-KV production path (plan + persistent kernel + merge) is checked
  on config 1 in full, on paged (page_size 16) batches, and with CTA counts
  that force every request to be cut.
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import TOL, HeadConfig, max_abs, rand, to_dev, to_np
from minisgl_b200 import workloads as W
from oracle import attention as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("hq,hkv,d", [(16, 8, 128), (32, 8, 128), (8, 8, 64), (16, 2, 256)])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_paged_decode_kernel(hq, hkv, d, dtype):
    import torch

    from minisgl_b200.attention import paged_decode_attention

    rng = np.random.default_rng(0)
    N, B = 4096, 7
    k_pool = rand(rng, (N, hkv, d), dtype)
    v_pool = rand(rng, (N, hkv, d), dtype)
    q = rand(rng, (B, hq, d), dtype)
    lens = [1, 2, 17, 31, 32, 33, 700]
    perm = rng.permutation(N).astype(np.int32)
    per_req, off = [], 0
    for n in lens:
        per_req.append(perm[off:off + n])
        off += n
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    indices = np.concatenate(per_req).astype(np.int32)
    scale = d ** -0.5
    out = paged_decode_attention(to_dev(q, dtype), to_dev(k_pool, dtype), to_dev(v_pool, dtype),
                                 torch.from_numpy(indptr).cuda(), torch.from_numpy(indices).cuda(),
                                 torch.tensor([scale], dtype=torch.float32))
    torch.cuda.synchronize()
    ref = O.reference_decode_per_request(q, k_pool, v_pool, per_req, scale)
    err = max_abs(to_np(out), ref)
    assert err <= TOL[dtype], f"max abs err {err}"


def _pool(B_slots, Hkv, D, dtype, rng, layers=1):
    import torch

    from minisgl_b200.kvcache import MHAKVCache
    from helpers import torch_dtype

    kv = MHAKVCache(layers, B_slots, Hkv, D, torch_dtype(dtype))
    host_k, host_v = [], []
    for l in range(layers):
        k = rand(rng, (B_slots, Hkv, D), dtype)
        v = rand(rng, (B_slots, Hkv, D), dtype)
        kv.k[l].copy_(torch.from_numpy(k))
        kv.v[l].copy_(torch.from_numpy(v))
        host_k.append(k)
        host_v.append(v)
    return kv, host_k, host_v


def _run_backend_decode(pb: W.PagedBatch, Hq, Hkv, D, dtype, num_ctas=None, seed=0):
    import torch

    from minisgl_b200.attention import B200AttnBackend

    rng = np.random.default_rng(seed)
    kv, hk, hv = _pool(pb.num_slots, Hkv, D, dtype, rng)
    be = B200AttnBackend(HeadConfig(Hq, Hkv, D), kv, pb.page_table, page_size=pb.page_size)
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens, num_ctas=num_ctas)
    q = rand(rng, (pb.batch_size, Hq, D), dtype)
    out = be.forward_decode(to_dev(q, dtype), 0, meta)
    torch.cuda.synchronize()
    idx, mask = O.naive_prepare_decode(pb.page_table, pb.rows, pb.lens)
    ref = O.naive_forward_decode(q, hk[0], hv[0], idx, mask, D ** -0.5)
    return to_np(out), ref, meta


@pytest.mark.parametrize("num_ctas", [None, 1, 5, 64, 600])
def test_config1_split_decode_fp32(num_ctas):
    """Config 1 (B=8, 16/8/128, fp32, page_size 1, N=16384) through the production path."""
    pb = W.config1_batch(seed=0)
    out, ref, meta = _run_backend_decode(pb, 16, 8, 128, "float32", num_ctas=num_ctas)
    if num_ctas and num_ctas >= 64:
        assert meta.n_partials > 0  # every request is cut at least once
    err = max_abs(out, ref)
    assert err <= TOL["float32"], err


@pytest.mark.parametrize("hq,hkv,d", [(16, 8, 128), (32, 8, 128), (8, 2, 64)])
@pytest.mark.parametrize("P", [1, 16])
@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_paged_split_decode(hq, hkv, d, P, dtype):
    rng = np.random.default_rng(11)
    lens = rng.integers(1, 1500, size=19)
    lens[:6] = [1, 2, 15, 16, 17, 33]
    pb = W.allocate_pages(lens, 65536, P, rng)
    for nc in (None, 7, 300):
        out, ref, _ = _run_backend_decode(pb, hq, hkv, d, dtype, num_ctas=nc, seed=3)
        err = max_abs(out, ref)
        assert err <= TOL[dtype], (nc, err)


@pytest.mark.parametrize("hq,hkv", [(32, 4), (16, 4), (64, 8), (32, 8), (64, 16)])
@pytest.mark.parametrize("P", [16, 64])
def test_tensor_core_decode_shapes(hq, hkv, P):
    """The tensor-core decode (decode_mma_kernel, bf16, D = 128, G = 4 or 8, Hkv 4 or 8,
    page size >= 16): every kernel instance and ring depth it has, ragged last pages, pages
    of 64 slots (16-token stages starting inside a page), forced splits and merges; Hkv 16
    (64q/16kv) is served by decode_kernel and must agree the same way."""
    rng = np.random.default_rng(13)
    lens = rng.integers(1, 2500, size=21)
    lens[:7] = [1, 2, 15, 16, 17, 63, 65]
    pb = W.allocate_pages(lens, 65536, P, rng)
    for nc in (None, 9, 400):
        out, ref, meta = _run_backend_decode(pb, hq, hkv, 128, "bfloat16", num_ctas=nc, seed=4)
        err = max_abs(out, ref)
        assert err <= TOL["bfloat16"], (nc, err)
        if nc == 400:
            assert meta.n_partials > 0


def test_config2_shape_decode_bf16():
    """Config 2 shapes (B=128, 16/8/128, page 16, pool 262144, fragmented pages), one layer."""
    pb = W.config2_batch(seed=0)
    out, ref, meta = _run_backend_decode(pb, 16, 8, 128, "bfloat16")
    err = max_abs(out, ref)
    assert err <= TOL["bfloat16"], err


def test_decode_watchdog_clear():
    """No bounded wait gave up during the tests above."""
    import ctypes

    import torch

    from minisgl_b200 import _native as nat

    code = ctypes.c_int(-1)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert code.value == 0


def test_decode_cuda_graph_replay_with_refreshed_metadata():
    """The decode path is capturable: launches are stream-ordered and allocation-free.

    A graph captured once replays with new q values (copied into the captured
    buffer) and metadata rebuilt in place by refresh_decode_metadata.
    """
    import torch

    from minisgl_b200.attention import B200AttnBackend

    rng = np.random.default_rng(21)
    Hq, Hkv, D, P = 16, 8, 128, 16
    lens = rng.integers(1, 900, size=23)
    pb = W.allocate_pages(lens, 32768, P, rng)
    kv, hk, hv = _pool(pb.num_slots, Hkv, D, "bfloat16", rng)
    be = B200AttnBackend(HeadConfig(Hq, Hkv, D), kv, pb.page_table, page_size=P)
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens)
    q_buf = to_dev(rand(rng, (len(lens), Hq, D), "bfloat16"), "bfloat16")
    be.forward_decode(q_buf, 0, meta)  # warm-up outside capture
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = be.forward_decode(q_buf, 0, meta)
    idx, mask = O.naive_prepare_decode(pb.page_table, pb.rows, pb.lens)
    for trial in range(2):
        q = rand(rng, (len(lens), Hq, D), "bfloat16")
        q_buf.copy_(to_dev(q, "bfloat16"))
        be.refresh_decode_metadata(meta, pb.rows, pb.lens)
        g.replay()
        torch.cuda.synchronize()
        ref = O.naive_forward_decode(q, hk[0], hv[0], idx, mask, D ** -0.5)
        assert max_abs(to_np(out), ref) <= TOL["bfloat16"], trial


@pytest.mark.parametrize("num_ctas", [None, 37])
def test_long_context_decode_qwen3_8b_shape(num_ctas):
    """Config-5 shape (32q/8kv/128, bf16, page 16) with contexts up to 32K tokens,
    split across many CTAs; oracle: per-request contiguous SDPA (tests/test_attention.py:10-16)."""
    rng = np.random.default_rng(5)
    lens = np.array([32768, 20011, 5, 4097])
    pb = W.allocate_pages(lens, 65536, 16, rng)
    out, _, meta = _run_backend_decode_ref(pb, 32, 8, 128, "bfloat16", num_ctas)
    assert meta.n_partials > 0
    assert out <= TOL["bfloat16"], out


def test_config5_decode_with_131072_token_request_and_200_partials():
    """Config 5 (Qwen3-8B attention 32q/8kv/128, bf16, page 16, contexts log-uniform in
    [1024, 131072]): the first 24 requests of the benchmark's seeded lengths with request 0
    set to the 131,072-token maximum, planned over 296 CTAs so that more than 200 split
    partials are written and merged. Oracle: the reference's per-request SDPA
    (tests/test_attention.py:10-16 form) in float32 torch on the CPU."""
    import torch

    from minisgl_b200 import MHAKVCache
    from minisgl_b200.attention import B200AttnBackend

    lens = W.config5_lens(seed=0)[:24].copy()
    lens[0] = 131072
    rng = np.random.default_rng(12)
    P, Hq, Hkv, D = 16, 32, 8, 128
    pages = int(((lens + P - 1) // P).sum())
    pb = W.allocate_pages(lens, (pages + 64) * P, P, rng)
    gen = torch.Generator(device="cuda").manual_seed(12)
    kv = MHAKVCache(1, pb.num_slots, Hkv, D, torch.bfloat16)
    kv.k[0].normal_(generator=gen)
    kv.v[0].normal_(generator=gen)
    q = torch.randn((len(lens), Hq, D), device="cuda", generator=gen).to(torch.bfloat16)
    be = B200AttnBackend(HeadConfig(Hq, Hkv, D), kv, pb.page_table, page_size=P)
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens, num_ctas=296)
    assert meta.n_partials >= 200, meta.n_partials
    out = be.forward_decode(q, 0, meta).float().cpu()
    torch.cuda.synchronize()
    kh, vh, qh = kv.k[0].cpu(), kv.v[0].cpu(), q.float().cpu()
    G = Hq // Hkv
    worst = 0.0
    for b, L in enumerate(lens.tolist()):
        sel = torch.from_numpy(pb.page_table[b, :L].astype(np.int64))
        k = kh[sel].float().permute(1, 0, 2)  # [Hkv, L, D]
        v = vh[sel].float().permute(1, 0, 2)
        s = torch.matmul(qh[b].view(Hkv, G, D), k.transpose(1, 2)) * D ** -0.5
        o = torch.matmul(torch.softmax(s, dim=-1), v).reshape(Hq, D)
        worst = max(worst, float((out[b] - o).abs().max()))
    assert worst <= TOL["bfloat16"], worst


def _run_backend_decode_ref(pb, Hq, Hkv, D, dtype, num_ctas):
    import torch

    from minisgl_b200.attention import B200AttnBackend

    rng = np.random.default_rng(9)
    kv, hk, hv = _pool(pb.num_slots, Hkv, D, dtype, rng)
    be = B200AttnBackend(HeadConfig(Hq, Hkv, D), kv, pb.page_table, page_size=pb.page_size)
    meta = be.decode_metadata_from_lens(pb.rows, pb.lens, num_ctas=num_ctas)
    q = rand(rng, (pb.batch_size, Hq, D), dtype)
    out = to_np(be.forward_decode(to_dev(q, dtype), 0, meta))
    torch.cuda.synchronize()
    per_req = [pb.page_table[b, : int(pb.lens[b])] for b in range(pb.batch_size)]
    ref = O.reference_decode_per_request(q.astype(np.float32), hk[0], hv[0], per_req, D ** -0.5)
    return max_abs(out, ref), None, meta
