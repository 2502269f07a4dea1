"""The engine harness end to end on the GPU.

* fp32: greedy tokens of a small random-init Qwen3 through the full harness
  (chunked prefill, radix prefix reuse, paging, overlap scheduling, decode
  CUDA graphs with padded buckets, the B200 attention kernels) are identical
  to the float64 full-recompute oracle (oracle/engine.py) -- the config-4
  parity check at test size.
* bf16: a config-4-shaped run (random prompts, ignore_eos) produces exactly
  max_tokens per request and leaves every KV page free or in the prefix cache.
"""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _prompts(rng):
    a = rng.integers(0, 500, 200).astype(np.int32)
    return [
        a,
        rng.integers(0, 500, 180).astype(np.int32),
        np.concatenate([a[:160], rng.integers(0, 500, 40).astype(np.int32)]),  # shares 10 pages with a
        rng.integers(0, 500, 30).astype(np.int32),
        rng.integers(0, 500, 520).astype(np.int32),  # chunked over three prefill steps
        np.concatenate([a[:96], rng.integers(0, 500, 10).astype(np.int32)]),
        rng.integers(0, 500, 1).astype(np.int32),  # a one-token prompt
    ]


@pytest.mark.parametrize("overlap,graphs,device_meta",
                         [(True, True, True), (False, True, True), (True, False, True), (True, True, False)])
def test_engine_fp32_tokens_match_oracle(overlap, graphs, device_meta):
    """Greedy tokens identical to the fp64 recompute oracle, with and without overlap
    scheduling, decode CUDA graphs and the device-built decode metadata."""
    import torch

    from minisgl_b200.core import SamplingParams
    from minisgl_b200.engine import LLM, EngineConfig, tiny_spec
    from oracle.engine import OracleQwen3

    rng = np.random.default_rng(4)
    prompts = _prompts(rng)
    max_tokens = [int(x) for x in rng.integers(8, 20, len(prompts))]
    cfg = EngineConfig(spec=tiny_spec(num_layers=2, vocab_size=500), dtype="float32", max_running_req=4,
                       page_size=16, num_tokens=8192, max_extend_tokens=256, overlap_scheduling=overlap,
                       cuda_graph_max_bs=4 if graphs else 0, device_metadata=device_meta)
    llm = LLM(cfg)
    outs = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in max_tokens])
    torch.cuda.synchronize()
    got = [o["token_ids"] for o in outs]
    assert [len(g) for g in got] == max_tokens
    want = OracleQwen3(llm.engine.model).generate(prompts, max_tokens)
    assert got == want
    assert llm.num_prefix_hit_tokens > 0  # the shared prefixes were served from the radix cache
    llm.cache.check_integrity()
    llm.engine.shutdown()


# The engine configurations of the reference's end-to-end parity test (tests/test_e2e.py:40-46)
# that do not name one of its MLX backends, plus its default page size 1 (engine/config.py:12).
REFERENCE_E2E_CONFIGS = {
    "chunked_prefill_16": dict(max_extend_tokens=16),
    "page_size_4": dict(page_size=4),
    "page_size_1": dict(page_size=1),
    "naive_cache": dict(cache_type="naive"),
}


@pytest.mark.parametrize("name", list(REFERENCE_E2E_CONFIGS))
def test_engine_fp32_reference_e2e_configs_two_rounds(name):
    """As the reference's test_greedy_matches_mlx_lm (tests/test_e2e.py:49-58): each config
    generates the same prompts twice, the second round served from the radix cache where
    there is one, and both rounds' greedy tokens equal the float64 recompute oracle."""
    import torch

    from minisgl_b200.core import SamplingParams
    from minisgl_b200.engine import LLM, EngineConfig, tiny_spec
    from oracle.engine import OracleQwen3

    rng = np.random.default_rng(6)
    prompts = _prompts(rng)
    max_tokens = [int(x) for x in rng.integers(8, 20, len(prompts))]
    base = dict(spec=tiny_spec(num_layers=2, vocab_size=500), dtype="float32", max_running_req=4, page_size=16,
                num_tokens=8192, max_extend_tokens=256, cuda_graph_max_bs=4)
    llm = LLM(EngineConfig(**{**base, **REFERENCE_E2E_CONFIGS[name]}))
    want = OracleQwen3(llm.engine.model).generate(prompts, max_tokens)
    hits = []
    for round_ in range(2):
        before = llm.num_prefix_hit_tokens
        outs = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in max_tokens])
        torch.cuda.synchronize()
        assert [o["token_ids"] for o in outs] == want, (name, round_)
        hits.append(llm.num_prefix_hit_tokens - before)
    if name == "naive_cache":
        assert hits == [0, 0]
    else:
        assert hits[1] > hits[0]  # the second round reuses the first round's prompts
    llm.cache.check_integrity()
    assert llm.table.available_size == 4
    llm.engine.shutdown()


def test_engine_bf16_config4_shape_runs_clean():
    import ctypes

    import torch

    from minisgl_b200 import _native as nat
    from minisgl_b200.core import SamplingParams
    from minisgl_b200.engine import LLM, EngineConfig, qwen3_0_6b_spec

    rng = np.random.default_rng(1)
    n = 24
    prompts = [rng.integers(0, 10000, int(rng.integers(100, 400))).astype(np.int32) for _ in range(n)]
    max_tokens = [int(x) for x in rng.integers(16, 64, n)]
    cfg = EngineConfig(spec=qwen3_0_6b_spec(), dtype="bfloat16", max_running_req=16, page_size=16,
                       num_tokens=16384, max_extend_tokens=1024)
    llm = LLM(cfg)
    outs = llm.generate(prompts, [SamplingParams(max_tokens=m, ignore_eos=True) for m in max_tokens])
    assert [len(o["token_ids"]) for o in outs] == max_tokens
    assert all(0 <= t < 151936 for o in outs for t in o["token_ids"])
    assert llm.num_output_tokens == sum(max_tokens)
    llm.cache.check_integrity()
    assert llm.table.available_size == 16
    code = ctypes.c_int(-1)
    nat.call("b2a_device_error", torch.cuda.current_stream().cuda_stream, ctypes.byref(code))
    assert code.value == 0
    llm.engine.shutdown()


def _tiny_llm(overlap=True):
    from minisgl_b200.engine import LLM, EngineConfig, tiny_spec

    cfg = EngineConfig(spec=tiny_spec(num_layers=2, vocab_size=500), dtype="float32", max_running_req=4,
                       page_size=16, num_tokens=8192, max_extend_tokens=256, overlap_scheduling=overlap,
                       cuda_graph_max_bs=4)
    return LLM(cfg)


@pytest.mark.parametrize("overlap", [True, False])
def test_engine_exact_max_tokens(overlap):
    """1, 2, 3 and 7 new tokens exactly, with and without overlap scheduling (where a
    request finishing one step earlier has already been put into the next batch)."""
    from minisgl_b200.core import SamplingParams

    rng = np.random.default_rng(9)
    lens = [1, 2, 3, 7]
    prompts = [rng.integers(0, 500, 20).astype(np.int32) for _ in lens]
    llm = _tiny_llm(overlap)
    outs = llm.generate(prompts, [SamplingParams(max_tokens=n, ignore_eos=True) for n in lens])
    assert [len(o["token_ids"]) for o in outs] == lens
    llm.cache.check_integrity()
    assert llm.table.available_size == 4
    llm.engine.shutdown()


def test_engine_stops_at_eos_and_returns_resources():
    """A request stops at the first EOS token, which is not in its output; requests
    with ignore_eos run to max_tokens; every page and table row is returned."""
    from minisgl_b200.core import SamplingParams

    rng = np.random.default_rng(5)
    prompts = [rng.integers(0, 500, int(n)).astype(np.int32) for n in (40, 17, 64)]
    llm = _tiny_llm()
    free_run = [o["token_ids"] for o in llm.generate(prompts, [SamplingParams(max_tokens=12, ignore_eos=True)] * 3)]
    llm.engine.shutdown()
    eos = free_run[0][4]  # request 0 meets it at its fifth token (or earlier)
    llm = _tiny_llm()
    llm.eos_token_ids = {eos}
    sps = [SamplingParams(max_tokens=12), SamplingParams(max_tokens=12), SamplingParams(max_tokens=12, ignore_eos=True)]
    outs = [o["token_ids"] for o in llm.generate(prompts, sps)]
    for i in range(2):
        want = free_run[i][: free_run[i].index(eos)] if eos in free_run[i] else free_run[i]
        assert outs[i] == want
    assert outs[2] == free_run[2]
    llm.cache.check_integrity()
    assert llm.table.available_size == 4
    llm.engine.shutdown()
