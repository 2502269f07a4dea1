"""End-to-end parity through the reference-facing plugin surface.

Drives the calls the reference's scheduler and model make -- Context,
create_attention_backend("b200", ...), backend.prepare_metadata(batch),
AttentionLayer(q, k, v) per layer, Req.complete_one() -- over a chunked
prefill with a prefix hit followed by decode steps, and compares every layer
output with the oracle running the reference's naive path on the same seeded
inputs (layers.py:103-111, attention/base.py, attention/naive.py).
"""

from __future__ import annotations

import numpy as np
import pytest

from helpers import TOL, HeadConfig, max_abs, rand, to_dev, to_np, torch_dtype
from oracle import attention as O

pytestmark = pytest.mark.gpu


class _Alloc:
    """Page allocator with the reference's contract (scheduler/cache.py:53-72)."""

    def __init__(self, num_slots, P, rng):
        self.P = P
        self.free = list(rng.permutation(num_slots // P) * P)

    def allocate(self, table, req):
        P = self.P
        first, last = -(-req.cached_len // P), -(-req.device_len // P)
        for p in range(first, last):
            s = self.free.pop()
            table[req.table_idx, p * P:(p + 1) * P] = np.arange(s, s + P)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("P", [1, 16])
def test_prefill_prefix_decode_sequence(dtype, P):
    import torch

    from minisgl_b200 import (AttentionLayer, Batch, Context, MHAKVCache, Req, RotaryConfig,
                              create_attention_backend, set_global_ctx)
    from minisgl_b200.core import batch_positions_out_loc

    L, Hq, Hkv, D, N = 2, 16, 8, 128, 8192
    rng = np.random.default_rng(0)
    rot = RotaryConfig(D, D, 1e6, 40960)
    table = np.zeros((4, 1024), np.int32)
    kv = MHAKVCache(L, N, Hkv, D, torch_dtype(dtype))
    ctx = Context(page_size=P)
    ctx.page_table = table
    ctx.kv_cache = kv
    be = create_attention_backend("b200", HeadConfig(Hq, Hkv, D), kv, table)
    ctx.attn_backend = be
    set_global_ctx(ctx)
    layers = [AttentionLayer(l, Hq, Hkv, D, rot) for l in range(L)]
    inv = layers[0].rotary.inv_freq_host
    hk = [np.zeros((N, Hkv, D), np.float32) for _ in range(L)]
    hv = [np.zeros((N, Hkv, D), np.float32) for _ in range(L)]
    alloc = _Alloc(N, P, rng)

    def step(batch):
        for r in batch.reqs:
            alloc.allocate(table, r)
        pos, loc = batch_positions_out_loc(batch, table)
        batch.positions = torch.from_numpy(pos).cuda()
        batch.out_loc = torch.from_numpy(loc).cuda()
        be.prepare_metadata(batch)
        T = len(pos)
        for l in range(L):
            q = rand(rng, (T, Hq, D), dtype)
            k = rand(rng, (T, Hkv, D), dtype)
            v = rand(rng, (T, Hkv, D), dtype)
            with ctx.forward_batch(batch):
                o = layers[l](to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype))
            torch.cuda.synchronize()
            qr = O.rope(q, pos, D, inv, 1.0, dtype)
            kr = O.rope(k, pos, D, inv, 1.0, dtype)
            O.store_kv(hk[l], hv[l], kr, v, loc)
            if batch.is_prefill:
                meta = O.prepare_prefill(table, [r.table_idx for r in batch.reqs],
                                         [r.cached_len for r in batch.reqs], [r.device_len for r in batch.reqs])
                ref = O.forward_prefill(qr, kr, v, hk[l], hv[l], meta, D ** -0.5)
            else:
                idx, mask = O.naive_prepare_decode(table, [r.table_idx for r in batch.reqs],
                                                   [r.device_len for r in batch.reqs])
                ref = O.naive_forward_decode(qr, hk[l], hv[l], idx, mask, D ** -0.5)
            assert o.shape == (T, Hq * D)
            err = max_abs(to_np(o).reshape(T, Hq, D), ref)
            assert err <= TOL[dtype], (batch.phase, l, err)
        for r in batch.reqs:
            r.complete_one()

    # prefill 1: A (40 tokens) and B0 (the 128-token prefix B will hit)
    A = Req(np.arange(40, dtype=np.int32), table_idx=0, cached_len=0, output_len=8)
    B0 = Req(np.arange(128, dtype=np.int32), table_idx=1, cached_len=0, output_len=1)
    step(Batch([A, B0], "prefill"))
    # prefill 2: B reuses B0's 128 cached slots (prefix hit, page aligned) and extends 172 tokens
    table[2, :128] = table[1, :128]
    B = Req(np.arange(300, dtype=np.int32), table_idx=2, cached_len=128, output_len=8)
    C = Req(np.arange(3, dtype=np.int32), table_idx=3, cached_len=0, output_len=8)
    step(Batch([B, C], "prefill"))
    # decode steps for A, B, C (A's first decode token was produced by prefill 1)
    for _ in range(3):
        step(Batch([A, B, C], "decode"))
    last = be.prepare_decode(Batch([A, B, C], "decode"))
    assert last.batch_size == 3
