"""The B200 attention backend (``--attn b200``).

Drop-in for the reference's backends (python/minisgl_mlx/attention/
{base,naive,metal}.py): same constructor ``(config, kv_cache, page_table)``,
same ``prepare_metadata`` / ``forward`` / ``prepare_decode`` /
``forward_decode`` contract, computed by the CUDA kernels of libb200attn.so:

* decode  -> ``b2a_decode``: persistent split-KV paged decode; split requests
  are merged inside the same launch (replaces metal.py:112-162 and naive.py:36-60)
* prefill -> ``b2a_extend``: ragged causal extend over the paged prefix
  (replaces base.py:70-105)

There is no CPU or library fallback: without the CUDA library or a GPU the
backend refuses to construct.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List

import numpy as np
import torch

from .. import _native as nat
from ..core import get_global_ctx
from ..kvcache.pool import current_stream_ptr, dtype_code
from .base import CHECK_METADATA, BaseAttnBackend, PinnedStager, paged_kv_indices


@dataclass
class B200DecodeMetadata:
    kv_indptr: torch.Tensor  # int32 [B+1] page CSR (device)
    kv_indices: torch.Tensor  # int32 [sum pages] page ids (device)
    kv_last_page_len: torch.Tensor  # int32 [B] (device)
    cta_indptr: torch.Tensor  # int32 [num_ctas+1] (device)
    segs: torch.Tensor  # int32 [n_segs, 4] (device)
    merge_indptr: torch.Tensor  # int32 [B+1] (device)
    n_partials: int
    num_ctas: int
    page_size: int
    batch_size: int
    workspace: torch.Tensor | None = None  # fixed split-partial workspace (CUDA-graph metadata)
    counts: torch.Tensor | None = None  # int32 [2] segments, split partials (device-built metadata)


@dataclass
class B200PrefillMetadata:
    last_indices: torch.Tensor  # int32 [B] (device): last token of each request in the packed batch
    q_offsets: List[int]  # [B+1] host, as reference PrefillMetadata
    qo_indptr: torch.Tensor  # int32 [B+1] (device)
    kv_indptr: torch.Tensor  # int32 [B+1] page CSR (device)
    kv_indices: torch.Tensor  # int32 page ids (device)
    kv_last_page_len: torch.Tensor  # int32 [B] (device)
    work: torch.Tensor  # int32 [n_work, 4] (device)
    n_work: int
    total_q: int
    page_size: int
    # set when the pool's page size is below what the tcgen05 extend needs: kv_indptr /
    # kv_indices / kv_last_page_len are then a CSR of 16-key groups and their first slots
    # (b2a_extend_groups); groups that are not one run of consecutive slots are packed
    # into a staging pool first (b2a_pack_kv) and their starts point there (>= num_slots)
    pack: "PackPlan | None" = None
    group_starts: bool = False


@dataclass
class PackPlan:
    """b2a_pack_kv row list: one 16-row staging page per group that is not a run."""

    src_kv_indices: torch.Tensor  # int32 [16 n] source slot of every staging row (device)
    n_groups: int
    out_slots: int  # 16 n


def _page_size() -> int:
    try:
        return int(get_global_ctx().page_size)
    except AssertionError:
        return 1


class B200AttnBackend(BaseAttnBackend):
    def __init__(self, config, kv_cache, page_table: np.ndarray, page_size: int | None = None) -> None:
        super().__init__(config, kv_cache, page_table)
        if not torch.cuda.is_available():
            raise RuntimeError("the b200 attention backend needs a CUDA device")
        self.device = kv_cache.device
        self.Hq = config.num_qo_heads
        self.Hkv = config.num_kv_heads
        self.D = config.head_dim
        self.dtype_code = dtype_code(kv_cache.dtype)
        self._page_size = page_size
        self._stager = PinnedStager()
        self._workspace = torch.empty(0, dtype=torch.uint8, device=self.device)
        self._stage: tuple | None = None  # packed K/V staging pools for small-page prefill
        n = nat.ctypes.c_int(0)
        with torch.cuda.device(self.device):
            nat.call("b2a_decode_num_ctas", self.Hq, self.Hkv, self.D, self.dtype_code, nat.ctypes.byref(n))
        self.num_ctas = n.value

    # ------------------------------------------------------------ helpers
    @property
    def page_size(self) -> int:
        return self._page_size if self._page_size is not None else _page_size()

    def _workspace_for(self, nbytes: int) -> torch.Tensor:
        # zero-filled once: the merge counters at its start must be zero before the
        # first decode call, and every call leaves them at zero again
        if self._workspace.numel() < nbytes:
            self._workspace = torch.zeros(max(nbytes, 2 * self._workspace.numel()), dtype=torch.uint8,
                                          device=self.device)
        return self._workspace

    # ------------------------------------------------------------ decode
    def prepare_decode(self, batch) -> B200DecodeMetadata:
        lens = np.array([r.device_len for r in batch.reqs], dtype=np.int64)
        rows = np.array([r.table_idx for r in batch.reqs], dtype=np.int64)
        return self.decode_metadata_from_lens(rows, lens)

    def decode_metadata_from_lens(self, rows: np.ndarray, lens: np.ndarray,
                                  num_ctas: int | None = None) -> B200DecodeMetadata:
        P = self.page_size
        kv_indptr, kv_indices, lpl = paged_kv_indices(self.page_table, rows, lens, P, check=CHECK_METADATA)
        nctas = num_ctas or self.num_ctas
        cta_indptr, segs, merge_indptr, n_partials = nat.decode_plan(kv_indptr, lpl, P, nctas)
        if CHECK_METADATA and kv_indices.size and int(kv_indices.max()) * P >= self.kv_cache.num_tokens:
            raise ValueError("kv_indices point past the end of the KV pool")
        dev = self._stager.upload([kv_indptr, kv_indices, lpl, cta_indptr, segs, merge_indptr], self.device)
        return B200DecodeMetadata(
            kv_indptr=dev[0], kv_indices=dev[1], kv_last_page_len=dev[2], cta_indptr=dev[3],
            segs=dev[4].view(-1, 4), merge_indptr=dev[5], n_partials=n_partials, num_ctas=nctas,
            page_size=P, batch_size=len(lens),
        )

    def refresh_decode_metadata(self, meta: B200DecodeMetadata, rows: np.ndarray, lens: np.ndarray) -> None:
        """Recompute the decode indices of a batch into ``meta``'s existing device tensors.

        For replaying a CUDA graph captured with ``meta``: the new plan must have the
        same sizes (same requests and page counts), otherwise ValueError.
        """
        P = meta.page_size
        kv_indptr, kv_indices, lpl = paged_kv_indices(self.page_table, rows, lens, P, check=CHECK_METADATA)
        cta_indptr, segs, merge_indptr, n_partials = nat.decode_plan(kv_indptr, lpl, P, meta.num_ctas)
        if n_partials > meta.n_partials:
            raise ValueError("refresh_decode_metadata: plan needs more split partials than the captured one")
        self._stager.upload([kv_indptr, kv_indices, lpl, cta_indptr, segs, merge_indptr], self.device,
                            out=[meta.kv_indptr, meta.kv_indices, meta.kv_last_page_len, meta.cta_indptr,
                                 meta.segs, meta.merge_indptr])

    # ------------------------------------------------------------ decode under CUDA graphs
    def alloc_decode_graph_metadata(self, batch_size: int, max_pages: int) -> B200DecodeMetadata:
        """Fixed-capacity decode metadata for a captured decode step of ``batch_size`` requests.

        Every per-step size the kernels need is read on the device (page CSR, the CTA
        plan, merge ranges), so a captured launch stays valid when
        ``fill_decode_graph_metadata`` rewrites these buffers in place. The split
        partials are laid out for the plan's worst case, ``batch_size + num_ctas``
        (each CTA boundary cuts at most one request), so any later plan fits.
        """
        dev, nc = self.device, self.num_ctas
        cap = batch_size + nc
        i32 = dict(dtype=torch.int32, device=dev)
        ws = torch.zeros(nat.decode_workspace_bytes(cap, self.Hq, self.D), dtype=torch.uint8, device=dev)
        return B200DecodeMetadata(
            kv_indptr=torch.zeros(batch_size + 1, **i32), kv_indices=torch.zeros(max(max_pages, 1), **i32),
            kv_last_page_len=torch.zeros(batch_size, **i32), cta_indptr=torch.zeros(nc + 1, **i32),
            segs=torch.zeros((cap + 1, 4), **i32), merge_indptr=torch.zeros(batch_size + 1, **i32),
            n_partials=cap, num_ctas=nc, page_size=self.page_size, batch_size=batch_size, workspace=ws,
            counts=torch.zeros(2, **i32),
        )

    def fill_decode_graph_metadata(self, meta: B200DecodeMetadata, rows: np.ndarray, lens: np.ndarray) -> None:
        """Plan ``len(rows) == meta.batch_size`` requests into ``meta``'s buffers (stream-ordered)."""
        P = meta.page_size
        kv_indptr, kv_indices, lpl = paged_kv_indices(self.page_table, rows, lens, P, check=CHECK_METADATA)
        cta_indptr, segs, merge_indptr, n_partials = nat.decode_plan(kv_indptr, lpl, P, meta.num_ctas)
        if len(kv_indptr) != meta.batch_size + 1:
            raise ValueError("fill_decode_graph_metadata: batch size differs from the captured one")
        if kv_indices.size > meta.kv_indices.numel() or segs.shape[0] > meta.segs.shape[0] or n_partials > meta.n_partials:
            raise ValueError("fill_decode_graph_metadata: plan exceeds the captured capacity")
        self._stager.upload(
            [kv_indptr, kv_indices, lpl, cta_indptr, segs, merge_indptr], self.device,
            out=[meta.kv_indptr, meta.kv_indices[: kv_indices.size], meta.kv_last_page_len, meta.cta_indptr,
                 meta.segs[: segs.shape[0]], meta.merge_indptr])

    def build_decode_metadata_device(self, meta: B200DecodeMetadata, page_table: torch.Tensor,
                                     rows: torch.Tensor, lens: torch.Tensor) -> None:
        """Fill ``meta`` (from ``alloc_decode_graph_metadata``) on the device (b2a_decode_metadata).

        ``page_table`` is a device int32 copy of the engine's page table, ``rows``
        and ``lens`` device int32 ``[meta.batch_size]``. Replaces the host CSR of
        attention/metal.py:145-152 and the host split plan; stream-ordered and
        capturable in a CUDA graph. The values equal ``fill_decode_graph_metadata``'s
        for the same rows and lengths.
        """
        B = meta.batch_size
        assert page_table.dtype == torch.int32 and page_table.is_contiguous() and page_table.dim() == 2
        assert rows.dtype == torch.int32 and lens.dtype == torch.int32 and rows.numel() >= B and lens.numel() >= B
        nat.call(
            "b2a_decode_metadata", page_table.data_ptr(), page_table.shape[0], page_table.shape[1],
            rows.data_ptr(), lens.data_ptr(), B, meta.page_size, meta.num_ctas,
            meta.kv_indptr.data_ptr(), meta.kv_indices.data_ptr(), meta.kv_indices.numel(),
            meta.kv_last_page_len.data_ptr(), meta.cta_indptr.data_ptr(), meta.segs.data_ptr(), meta.segs.shape[0],
            meta.merge_indptr.data_ptr(), meta.counts.data_ptr(), current_stream_ptr(self.device),
        )

    def forward_decode(self, q: torch.Tensor, layer_id: int, meta: B200DecodeMetadata) -> torch.Tensor:
        B = meta.batch_size
        assert q.shape == (B, self.Hq, self.D), q.shape
        q = q.contiguous()
        out = torch.empty_like(q)
        ws_bytes = nat.decode_workspace_bytes(meta.n_partials, self.Hq, self.D)
        ws = meta.workspace if meta.workspace is not None else self._workspace_for(ws_bytes)
        assert ws.numel() >= ws_bytes
        nat.call(
            "b2a_decode", q.data_ptr(), self.kv_cache.k_cache(layer_id).data_ptr(),
            self.kv_cache.v_cache(layer_id).data_ptr(), self.kv_cache.num_tokens, meta.kv_indices.data_ptr(),
            meta.page_size,
            meta.cta_indptr.data_ptr(), meta.segs.data_ptr(), meta.num_ctas, meta.merge_indptr.data_ptr(),
            meta.n_partials, B, self.Hq, self.Hkv, self.D, float(self.scale), ws.data_ptr(), ws.numel(),
            out.data_ptr(), self.dtype_code, current_stream_ptr(self.device),
        )
        return out

    # ------------------------------------------------------------ prefill / extend
    def _prepare_prefill(self, batch) -> B200PrefillMetadata:
        extend = np.array([r.extend_len for r in batch.reqs], dtype=np.int64)
        lens = np.array([r.device_len for r in batch.reqs], dtype=np.int64)
        rows = np.array([r.table_idx for r in batch.reqs], dtype=np.int64)
        return self.extend_metadata_from_lens(rows, lens, extend)

    def extend_metadata_from_lens(self, rows: np.ndarray, lens: np.ndarray,
                                  extend: np.ndarray) -> B200PrefillMetadata:
        P = self.page_size
        qo_indptr = np.zeros(len(extend) + 1, np.int32)
        np.cumsum(extend, out=qo_indptr[1:])
        kv_indptr, kv_indices, lpl = paged_kv_indices(self.page_table, rows, lens, P, check=CHECK_METADATA)
        tile_q = nat.extend_tile_q(self.Hq, self.Hkv, self.D, self.dtype_code, P)
        if P < self.PACK_PAGE:
            tile16 = nat.extend_tile_q(self.Hq, self.Hkv, self.D, self.dtype_code, self.PACK_PAGE)
            if tile16 != tile_q:  # the tensor-core kernel takes this shape in groups of 16 keys
                return self._grouped_extend_metadata(qo_indptr, np.asarray(lens, dtype=np.int64), kv_indptr,
                                                     kv_indices, P, tile16)
        work = nat.extend_plan(qo_indptr, kv_indptr, lpl, P, tile_q)
        last_indices = (qo_indptr[1:] - 1).astype(np.int32)
        dev = self._stager.upload([last_indices, qo_indptr, kv_indptr, kv_indices, lpl, work], self.device)
        return B200PrefillMetadata(
            last_indices=dev[0], q_offsets=qo_indptr.tolist(), qo_indptr=dev[1], kv_indptr=dev[2],
            kv_indices=dev[3], kv_last_page_len=dev[4], work=dev[5].view(-1, 4), n_work=int(work.shape[0]),
            total_q=int(qo_indptr[-1]), page_size=P,
        )

    PACK_PAGE = 16

    def _grouped_extend_metadata(self, qo_indptr, lens, src_indptr, src_indices, P, tile_q) -> B200PrefillMetadata:
        """Extend metadata for a pool whose page size is below 16 (b2a_extend_groups): the
        16-key groups of ``extend_key_groups``, their packed rows uploaded with the rest."""
        Q = self.PACK_PAGE
        group_indptr, starts, lpl, rows = extend_key_groups(lens, src_indptr, src_indices, P,
                                                            self.kv_cache.num_tokens, Q)
        n_packed = len(rows) // Q
        work = nat.extend_plan(qo_indptr, group_indptr, lpl, Q, tile_q)
        last_indices = (qo_indptr[1:] - 1).astype(np.int32)
        arrays = [last_indices, qo_indptr, group_indptr, starts, lpl, work]
        if n_packed:
            arrays.append(rows)
        dev = self._stager.upload(arrays, self.device)
        pack = PackPlan(src_kv_indices=dev[6], n_groups=n_packed, out_slots=Q * n_packed) if n_packed else None
        return B200PrefillMetadata(
            last_indices=dev[0], q_offsets=qo_indptr.tolist(), qo_indptr=dev[1], kv_indptr=dev[2],
            kv_indices=dev[3], kv_last_page_len=dev[4], work=dev[5].view(-1, 4), n_work=int(work.shape[0]),
            total_q=int(qo_indptr[-1]), page_size=Q, pack=pack, group_starts=True,
        )

    def _stage_for(self, slots: int):
        """Packed K/V staging pools of at least ``slots`` rows.

        Zero-initialised and only ever written with K/V rows, like the real pool: the
        tail of a request's last packed page (rows past its length) is multiplied by
        a softmax weight of exactly 0, which is only harmless for finite values.
        """
        if self._stage is None or self._stage[0].shape[0] < slots:
            n = max(slots, 0 if self._stage is None else 2 * self._stage[0].shape[0])
            self._stage = tuple(torch.zeros((n, self.Hkv, self.D), dtype=self.kv_cache.dtype, device=self.device)
                                for _ in range(2))
        return self._stage[0][:slots], self._stage[1][:slots]

    def _forward_prefill(self, q, k, v, layer_id: int, meta: B200PrefillMetadata) -> torch.Tensor:
        T = meta.total_q
        assert q.shape == (T, self.Hq, self.D), q.shape
        q = q.contiguous()
        out = torch.empty_like(q)
        B = len(meta.q_offsets) - 1
        k_pool, v_pool = self.kv_cache.k_cache(layer_id), self.kv_cache.v_cache(layer_id)
        num_slots = self.kv_cache.num_tokens
        if meta.group_starts:
            k_st = v_st = None
            stage_slots = 0
            if meta.pack is not None:
                pk = meta.pack
                k_st, v_st = self._stage_for(pk.out_slots)
                stage_slots = pk.out_slots
                nat.call(
                    "b2a_pack_kv", k_pool.data_ptr(), v_pool.data_ptr(), num_slots, None,
                    pk.src_kv_indices.data_ptr(), 1, None, None, pk.n_groups, pk.out_slots, self.Hkv, self.D,
                    self.dtype_code, k_st.data_ptr(), v_st.data_ptr(), pk.out_slots, current_stream_ptr(self.device),
                )
            nat.call(
                "b2a_extend_groups", q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), num_slots,
                None if k_st is None else k_st.data_ptr(), None if v_st is None else v_st.data_ptr(), stage_slots,
                meta.qo_indptr.data_ptr(), meta.kv_indptr.data_ptr(), meta.kv_indices.data_ptr(),
                meta.kv_last_page_len.data_ptr(), meta.work.data_ptr(), meta.n_work, T, B, self.Hq, self.Hkv,
                self.D, float(self.scale), out.data_ptr(), self.dtype_code, current_stream_ptr(self.device),
            )
            return out
        nat.call(
            "b2a_extend", q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), num_slots, meta.qo_indptr.data_ptr(),
            meta.kv_indptr.data_ptr(), meta.kv_indices.data_ptr(), meta.kv_last_page_len.data_ptr(),
            meta.page_size, meta.work.data_ptr(), meta.n_work, T, B, self.Hq, self.Hkv, self.D,
            float(self.scale), out.data_ptr(), self.dtype_code, current_stream_ptr(self.device),
        )
        return out


def extend_key_groups(lens, src_indptr, src_indices, P: int, num_slots: int, Q: int = 16):
    """Keys of every request in groups of Q = 16 for b2a_extend_groups, over a pool whose page
    size P is below 16.

    Group j of request b covers keys [16 j, 16 j + 16). A group whose slots are one run of
    consecutive slots that lies wholly inside the pool (what a fresh free list hands a
    prompt) is read in place: its start is its first slot. Every other group is packed into
    a 16-row page of a staging pool, in group order, and starts at num_slots + 16 * page.

    lens [B] keys per request; src_indptr [B+1] / src_indices the page CSR of the pool
    (page ids, P slots each). Returns int32 arrays: group_indptr [B+1], starts [groups],
    the key count of each request's last group [B] (0 for an empty request), and the
    source slot of every staging row [16 * packed groups] (row 16 k + i of packed group k;
    rows past a short last group repeat its last slot and are never attended).
    """
    lens = np.asarray(lens, dtype=np.int64)
    B = len(lens)
    tok_indptr = np.zeros(B + 1, np.int64)
    np.cumsum(lens, out=tok_indptr[1:])
    T_kv = int(tok_indptr[-1])
    if T_kv >= 2 ** 31:
        raise ValueError("grouped extend: more than 2^31 KV rows in one batch")
    req = np.repeat(np.arange(B), lens)
    pos = np.arange(T_kv, dtype=np.int64) - tok_indptr[req]
    src_indptr = np.asarray(src_indptr, dtype=np.int64)
    src_indices = np.asarray(src_indices, dtype=np.int64)
    tok = src_indices[src_indptr[req] + pos // P] * P + pos % P  # slot of every key, in key order
    ngroups = (lens + Q - 1) // Q
    group_indptr = np.zeros(B + 1, np.int64)
    np.cumsum(ngroups, out=group_indptr[1:])
    G = int(group_indptr[-1])
    gid = group_indptr[req] + pos // Q
    gfirst = np.zeros(G, np.int64)  # key index of each group's first key
    gfirst[gid[pos % Q == 0]] = np.nonzero(pos % Q == 0)[0]
    greq = np.repeat(np.arange(B), ngroups)
    glen = np.minimum(Q, lens[greq] - Q * (np.arange(G) - group_indptr[greq]))
    run_ok = tok == tok[gfirst[gid]] + pos % Q
    group_ok = np.logical_and.reduceat(run_ok, gfirst) if G else np.zeros(0, bool)
    # a run is read in place only inside the pool: any other slot goes through the
    # packer, whose bounds check reports it (a start >= num_slots means the staging pool)
    if G:
        group_ok &= (tok[gfirst] >= 0) & (tok[gfirst] + glen <= num_slots)
    packed = np.nonzero(~group_ok)[0]
    n_packed = len(packed)
    starts = np.where(group_ok, tok[gfirst] if G else 0, 0).astype(np.int64)
    starts[packed] = num_slots + Q * np.arange(n_packed, dtype=np.int64)
    if G and starts.max() >= 2 ** 31:
        raise ValueError("grouped extend: staging slots past 2^31")
    lpl = np.where(ngroups > 0, lens - (ngroups - 1) * Q, 0).astype(np.int32)
    rows = gfirst[packed][:, None] + np.minimum(np.arange(Q)[None, :], glen[packed][:, None] - 1)
    return (group_indptr.astype(np.int32), starts.astype(np.int32), lpl,
            tok[rows.reshape(-1)].astype(np.int32))


def paged_decode_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                           kv_indptr: torch.Tensor, kv_indices: torch.Tensor, scale) -> torch.Tensor:
    """Same call as the reference's ``paged_decode_attention`` (attention/metal.py:112-131).

    q ``[B, Hq, D]``; pools ``[N, Hkv, D]``; kv_indptr int32 ``[B+1]`` token CSR;
    kv_indices int32 slots; scale a float or a 1-element tensor. One CTA per request
    (``b2a_paged_decode``), no workspace.
    """
    B, Hq, D = q.shape
    Hkv = k_pool.shape[1]
    assert D % 32 == 0 and Hq % Hkv == 0
    assert kv_indptr.dtype == torch.int32 and kv_indices.dtype == torch.int32
    assert k_pool.is_contiguous() and v_pool.is_contiguous() and k_pool.shape == v_pool.shape
    if isinstance(scale, torch.Tensor):
        scale = float(scale.reshape(-1)[0].item())
    q = q.contiguous()
    out = torch.empty_like(q)
    nat.call(
        "b2a_paged_decode", q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr(), k_pool.shape[0], kv_indptr.data_ptr(),
        kv_indices.data_ptr(), B, Hq, Hkv, D, float(scale), out.data_ptr(), dtype_code(q.dtype),
        current_stream_ptr(q.device),
    )
    return out


def page_table_scatter(page_table: torch.Tensor, rows: torch.Tensor, cols: torch.Tensor, values: torch.Tensor) -> None:
    """``page_table[rows[i], cols[i]] = values[i]`` on the device (b2a_page_table_scatter).

    Applies the slots a step allocated on the host to a device copy of the page
    table (the input of ``build_decode_metadata_device``). All int32, same device.
    """
    assert page_table.dtype == torch.int32 and page_table.is_contiguous() and page_table.dim() == 2
    n = rows.numel()
    assert cols.numel() == n and values.numel() == n
    for t in (rows, cols, values):
        assert t.dtype == torch.int32 and t.is_contiguous()
    nat.call("b2a_page_table_scatter", page_table.data_ptr(), page_table.shape[0], page_table.shape[1],
             rows.data_ptr(), cols.data_ptr(), values.data_ptr(), n, current_stream_ptr(page_table.device))
