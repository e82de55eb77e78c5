"""The static KV cache (PIMStaticKVCache.update / read_tile) and the attention masks.

Pinned by the reference itself (tests/golden/kv_cache_golden.json, written by
tests/golden/make_golden.py from memory/kv_layout.py:167-252 on its NumpyBackend):
the same seeded updates must leave byte-identical arenas and tiles, the masks must be
byte-identical, and decode attention over tiles read back (tile 6 over max_seq 16, not a
multiple) must equal the reference's and single-card PyTorch.  The CPU tests run on the
oracle HAL; the GPU test runs the same cache on the B200 HAL's arenas.
"""

from __future__ import annotations

import json
import sys

import numpy as np
import pytest

from helpers import GOLDEN, sha

sys.path.insert(0, str(GOLDEN))
import make_golden as mg  # noqa: E402  (seeded steps and the tiled attention of the fixture)

GOLD = json.loads((GOLDEN / "kv_cache_golden.json").read_text())


def _specs():
    from memory.kv_layout import KVRegionSpec, build_kv_layout

    def spec(rank, heads):
        return build_kv_layout(KVRegionSpec(dpu_id=rank, layers=list(range(mg.KVC_LAYERS)), kv_heads=list(heads),
                                            q_heads_by_kv={h: [h] for h in heads}, max_seq=mg.KVC_MAX,
                                            head_dim=mg.KVC_HD, dtype_bytes=4, kv_base=0), align=64)

    return {0: spec(0, (0, 1)), 1: spec(1, (2, 3))}


def _fill(hal):
    from memory.kv_layout import PIMStaticKVCache

    specs = _specs()
    cache = PIMStaticKVCache(hal, specs, wram_budget_bytes=mg.KVC_TILE * mg.KVC_HD * 4)
    for layer, pos, by in mg.kv_cache_steps():
        cache.update(layer, pos, {r: {h: kv[0] for h, kv in d.items()} for r, d in by.items()},
                     {r: {h: kv[1] for h, kv in d.items()} for r, d in by.items()})
    return cache, specs


def _check_cache(hal):
    from memory.kv_layout import decode_mask

    cache, specs = _fill(hal)
    for r, s in specs.items():
        assert [[l, h, w, o] for (l, h, w), o in sorted(s.kv_off.items())] == GOLD["kv_off"][str(r)]
    n = GOLD["kv_allocated_bytes"]
    assert [sha(hal.read_local(r, 0, (n,), np.uint8)) for r in (0, 1)] == GOLD["arena_sha"]
    for key, (ks, vs) in GOLD["tiles"].items():
        layer, rank, h, s0 = map(int, key.split("/"))
        k, v = cache.read_tile(layer, rank, h, s0, min(s0 + mg.KVC_TILE, mg.KVC_MAX))
        assert (sha(k), sha(v)) == (ks, vs), key
    rng = np.random.default_rng(GOLD["attention_q_seed"])
    q = {h: rng.standard_normal(mg.KVC_HD).astype(np.float32) for h in range(4)}
    out = mg.kv_cache_attention(cache, cache.read_tile, 1, q, GOLD["attention_valid_len"], decode_mask)
    for h, ref in GOLD["attention"].items():
        np.testing.assert_allclose(out[int(h)], np.asarray(ref, np.float32), rtol=0, atol=1e-6)
    return cache, q, out


def test_kv_cache_matches_the_reference_on_the_oracle():
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    hal = NumpyBackend(NumpyBackendConfig(2, 1 << 16))
    _check_cache(hal)
    hal.close()


def test_tiled_decode_attention_matches_single_card_torch():
    import torch

    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    hal = NumpyBackend(NumpyBackendConfig(2, 1 << 16))
    _, q, out = _check_cache(hal)
    valid = GOLD["attention_valid_len"]
    rows = {h: [] for h in range(4)}
    for layer, pos, by in mg.kv_cache_steps():
        if layer == 1 and pos <= valid:
            for d in by.values():
                for h, kv in d.items():
                    rows[h].append(kv)
    for h in range(4):
        K = torch.tensor(np.stack([k for k, _ in rows[h]]))
        V = torch.tensor(np.stack([v for _, v in rows[h]]))
        ref = torch.softmax(K @ torch.tensor(q[h]) / np.sqrt(mg.KVC_HD), dim=0) @ V
        np.testing.assert_allclose(out[h], ref.numpy(), atol=1e-6)
    hal.close()


def test_masks_match_the_reference():
    from memory.kv_layout import decode_mask, prefill_mask

    for key, want in GOLD["prefill_mask_sha"].items():
        p, m = map(int, key.split("/"))
        assert sha(prefill_mask(p, m)) == want
    for key, want in GOLD["decode_mask_sha"].items():
        v, m = map(int, key.split("/"))
        assert sha(decode_mask(v, m)) == want


def test_cache_checks_positions_heads_and_tile_budget():
    from oracle.hal_numpy import NumpyBackend, NumpyBackendConfig

    hal = NumpyBackend(NumpyBackendConfig(2, 1 << 16))
    cache, _ = _fill(hal)
    with pytest.raises(KeyError):
        cache.read_tile(0, 0, 2, 0, 4)  # head 2 lives on rank 1
    with pytest.raises(ValueError):
        cache.read_tile(0, 0, 0, 10, 17)  # past max_seq
    with pytest.raises(ValueError):
        cache.read_tile(0, 0, 0, 0, mg.KVC_TILE + 1)  # over the staging budget
    bad = {0: {0: np.zeros(4, np.float32), 1: np.zeros(4, np.float32)},
           1: {2: np.zeros(4, np.float32), 3: np.zeros(4, np.float32)}}
    with pytest.raises(ValueError):
        cache.update(0, 0, bad, bad)  # rows of the wrong length
    hal.close()


@pytest.mark.gpu
def test_kv_cache_matches_the_reference_on_the_b200_hal():
    from backend.hal_cuda import CudaBackend, CudaBackendConfig

    hal = CudaBackend(CudaBackendConfig(2, 1 << 16))
    _check_cache(hal)
    hal.close()
