"""CPU replay of the decode attention's work items (go-infer_b200/csrc/attn.cuh
attn_partial_item and attn_heads_per_item; the per-layer launch in model.cu,
the item loop of the persistent kernel in layers.cu): for every grouping the
items cover each (query head, chunk) exactly once, each chunk's cache slot
is written by exactly one item, and the head counts chosen for config 5's
shapes under tensor parallelism are the ones the launches use."""
import pytest


def heads_per_item(kv_mul, n_kv_heads, splits, target):
    """attn_heads_per_item: kv_mul halved while the items number fewer than target."""
    hq = kv_mul
    while hq > 1 and hq % 2 == 0 and n_kv_heads * splits * (kv_mul // hq) < target:
        hq //= 2
    return hq


def per_layer_items(n_kv_heads, kv_mul, splits, hq):
    """The per-layer launch: grid (n_kv_heads * ng, splits), blockIdx.x = g * ng + hg."""
    ng = kv_mul // hq
    for bx in range(n_kv_heads * ng):
        for by in range(splits):
            yield bx // ng, by, bx % ng


def persistent_items(n_kv_heads, kv_mul, splits, hq):
    """The persistent kernel: item it = (g * ng + hg) * splits + c."""
    ng = kv_mul // hq
    for it in range(n_kv_heads * ng * splits):
        gh = it // splits
        yield gh // ng, it % splits, gh % ng


def check_cover(items, n_kv_heads, kv_mul, splits, hq):
    seen = {}
    writers = {}
    for g, c, hg in items:
        assert 0 <= g < n_kv_heads and 0 <= c < splits and 0 <= hg < kv_mul // hq
        h_first = g * kv_mul + hg * hq  # attn_partial_item's first query head
        for h in range(h_first, h_first + hq):
            assert (h, c) not in seen, f"head {h} chunk {c} twice"
            seen[(h, c)] = True
            assert h // kv_mul == g  # the item's heads belong to its kv head
        if hg == 0:  # the item that writes this step's slot of chunk c for kv head g
            writers[(g, c)] = writers.get((g, c), 0) + 1
    assert len(seen) == n_kv_heads * kv_mul * splits
    assert all(v == 1 for v in writers.values()) and len(writers) == n_kv_heads * splits


@pytest.mark.parametrize("n_kv_heads,kv_mul,splits,sms", [
    (8, 8, 18, 148), (4, 8, 18, 148), (2, 8, 18, 148), (1, 8, 18, 148),   # config 5 at TP 1/2/4/8
    (32, 1, 6, 148),                                                       # config 4 (no GQA)
    (2, 4, 3, 148), (1, 6, 5, 148), (3, 2, 1, 16), (1, 16, 2, 148),
])
def test_items_cover_every_head_and_chunk_once(n_kv_heads, kv_mul, splits, sms):
    for target in (2 * sms, sms // 2 + 1):  # per-layer kernel, persistent kernel
        hq = heads_per_item(kv_mul, n_kv_heads, splits, target)
        assert kv_mul % hq == 0
        check_cover(per_layer_items(n_kv_heads, kv_mul, splits, hq), n_kv_heads, kv_mul, splits, hq)
        check_cover(persistent_items(n_kv_heads, kv_mul, splits, hq), n_kv_heads, kv_mul, splits, hq)


def test_config5_groupings():
    """Config 5 (8 kv heads, 8 query heads each, 576 slots = 18 chunks) on
    148 SMs: the per-layer kernel gets at least two items per SM, the
    persistent kernel one round of items per CTA."""
    want = {1: (2, 576, 8, 144), 2: (1, 576, 4, 144), 4: (1, 288, 2, 144), 8: (1, 144, 1, 144)}
    for world, (hq_l, items_l, hq_p, items_p) in want.items():
        nkv = 8 // world
        hl = heads_per_item(8, nkv, 18, 2 * 148)
        hp = heads_per_item(8, nkv, 18, 148 // 2 + 1)
        assert (hl, nkv * 18 * (8 // hl)) == (hq_l, items_l)
        assert (hp, nkv * 18 * (8 // hp)) == (hq_p, items_p)
        assert items_p <= 148  # one round on the persistent kernel's CTAs
