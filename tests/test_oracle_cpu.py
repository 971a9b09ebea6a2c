"""Pins of the CPU oracle: against the reference's golden RoPE bytes, against independent
restatements (numpy) and against properties the mathematics guarantees."""
import json
import math
from pathlib import Path

import numpy as np

from hyperkernel_b200 import workload as W

GOLDEN = Path(__file__).parent / "golden" / "rope_windows.json"


def test_oracle_rope_matches_reference_fixture(orc):
    data = json.loads(GOLDEN.read_text())
    for t in data["tables"]:
        p = t["params"]
        rows = max(w["row"] for w in t["windows"]) + 8
        table = orc.rope_table(rows, p["dim"], p["base"], p["original_seq_len"], p["factor"],
                               p["beta_fast"], p["beta_slow"])
        for w in t["windows"]:
            want = bytes.fromhex(w["hex"])
            assert table[w["row"]:].tobytes()[:len(want)] == want, (t["name"], w["row"])


def test_e4m3_known_answers_and_numpy_agree(orc):
    known = {0.0: 0x00, 1.0: 0x38, -1.0: 0xB8, 448.0: 0x7E, 1000.0: 0x7E, -1e9: 0xFE,
             2.0 ** -9: 0x01, 2.0 ** -6: 0x08, 1.0625: 0x38, 1.1875: 0x3A, 0.0009765625: 0x00}
    for x, code in known.items():
        assert orc.f32_to_e4m3(x) == code, (x, hex(orc.f32_to_e4m3(x)))
    for v in range(256):
        if (v & 0x7F) == 0x7F:
            continue
        f = orc.e4m3_to_f32(v)
        assert orc.f32_to_e4m3(f) == v or (f == 0.0 and v in (0x00, 0x80))
    xs = W.Rng(5).normal(20000).astype(np.float32) * np.float32(50.0)
    ours = np.array([orc.f32_to_e4m3(float(x)) for x in xs], dtype=np.uint8)
    assert np.array_equal(ours, W.e4m3_encode(xs))
    assert np.allclose(W.e4m3_decode(ours), [orc.e4m3_to_f32(int(v)) for v in ours])


def test_sigmoid_is_accurate(orc):
    for x in np.linspace(-20, 20, 401):
        s = orc.sigmoid(float(x))
        assert abs(s - 1 / (1 + math.exp(-x))) <= 2e-7 * max(1.0, s), x


def test_pack_known_answer(orc):
    # lanes: idle, decode at 5, spec block of 3 at 62 (crosses a page of 64), prompt of 4 at 0
    bt = np.array([[0, 0], [7, 0], [3, 9], [4, 0]], np.int32)
    o = orc.pack([0, 1, 3, 4], [0, 5, 62, 0], bt, 64, 16, 16)
    assert o["err"] == 0 and o["num_tokens"] == 8
    assert o["cu_seqlens"].tolist() == [0, 0, 1, 4, 8]
    assert o["seq_lens"].tolist() == [0, 6, 65, 4]
    assert o["positions"][:8].tolist() == [5, 62, 63, 64, 0, 1, 2, 3]
    assert o["slot_mapping"][:8].tolist() == [7 * 64 + 5, 3 * 64 + 62, 3 * 64 + 63, 9 * 64,
                                              256, 257, 258, 259]
    assert o["token_lane"][:8].tolist() == [1, 2, 2, 2, 3, 3, 3, 3]
    assert o["active"][:4].tolist() == [3, 1, 2, 3]


def test_pack_flags_scratch_page_and_overflow(orc):
    bt = np.array([[0, 0]], np.int32)
    o = orc.pack([1], [3], bt, 64, 4, 4)
    assert o["err"] == 2 and o["slot_mapping"][0] == -1
    o = orc.pack([5], [0], np.array([[1]], np.int32), 64, 4, 4)
    assert o["err"] == 1


def test_permute_is_a_stable_sort(orc):
    rng = W.Rng(11)
    T, K, E = 37, 4, 9
    ids = rng.integers(0, E - 1, T * K).reshape(T, K).astype(np.int32)
    w = rng.uniform(T * K).astype(np.float32).reshape(T, K)
    off, tok, pw, inv = orc.permute(ids, w, E)
    pairs = sorted(range(T * K), key=lambda p: (ids.flat[p], p))
    assert [p // K for p in pairs] == tok.tolist()
    assert np.array_equal(inv[pairs], np.arange(T * K))
    assert off.tolist() == [0] + np.cumsum(np.bincount(ids.ravel(), minlength=E)).tolist()
    assert np.array_equal(pw[inv], w.ravel())


def test_route_matches_argsort(orc):
    rng = W.Rng(12)
    T, E, K = 64, 256, 8
    logits = rng.normal(T * E).astype(np.float32).reshape(T, E)
    bias = (rng.normal(E) * 0.1).astype(np.float32)
    ids, w = orc.route(logits, bias, K, 2.5)
    s = 1 / (1 + np.exp(-logits.astype(np.float64)))
    want = np.argsort(-(s + bias), axis=1, kind="stable")[:, :K]
    assert np.array_equal(ids, want)
    sel = np.take_along_axis(s, want, 1)
    assert np.allclose(w, sel / sel.sum(1, keepdims=True) * 2.5, rtol=1e-5)


def test_split_attention_merges_to_whole(orc):
    """LSE merge property: attention over [0, n) equals the merge of attention over a split."""
    lay = W.config2_layout(seed=4, lanes=3, lo=100, hi=700)
    inp = W.mla_inputs(lay, 16, seed=5)
    o = orc.pack(lay.new_rows, lay.context, lay.block_table, 64, lay.num_pages, lay.num_tokens)
    kw = dict(kv_bf16=inp["kv_cache"])
    T = lay.num_tokens
    full, lse = orc.mla_decode(inp["q"], lay.block_table, o["cu_seqlens"], o["positions"][:T], 64,
                               inp["scale"], **kw)
    cut = (lay.context // 3).astype(np.int32)
    a, la = orc.mla_decode(inp["q"], lay.block_table, o["cu_seqlens"], o["positions"][:T], 64,
                           inp["scale"], kv_begin=np.zeros(3, np.int32), kv_end=cut, **kw)
    b, lb = orc.mla_decode(inp["q"], lay.block_table, o["cu_seqlens"], o["positions"][:T], 64,
                           inp["scale"], kv_begin=cut, kv_end=np.full(3, 1 << 30, np.int32), **kw)
    m, lm = orc.lse_merge(np.stack([a.reshape(-1, 512), b.reshape(-1, 512)]),
                          np.stack([la.ravel(), lb.ravel()]))
    assert np.allclose(m, full.reshape(-1, 512), atol=2e-6)
    assert np.allclose(lm, lse.ravel(), atol=2e-6)


def test_mla_oracle_matches_numpy(orc):
    lay = W.config2_layout(seed=6, lanes=2, lo=60, hi=200)
    inp = W.mla_inputs(lay, 16, seed=7)
    o = orc.pack(lay.new_rows, lay.context, lay.block_table, 64, lay.num_pages, lay.num_tokens)
    T = lay.num_tokens
    got, lse = orc.mla_decode(inp["q"], lay.block_table, o["cu_seqlens"], o["positions"][:T], 64,
                              inp["scale"], kv_bf16=inp["kv_cache"])
    q = W.bf16_bits_to_f32(inp["q"]).astype(np.float64)
    for t in range(T):
        b = t
        pos = int(o["positions"][t])
        slots = [int(lay.block_table[b, p // 64]) * 64 + p % 64 for p in range(pos + 1)]
        k = W.bf16_bits_to_f32(W.latent_rows(inp["kv_cache"], slots)).astype(np.float64)
        s = q[t] @ k.T * inp["scale"]
        p = np.exp(s - s.max(1, keepdims=True))
        want = (p @ k[:, :512]) / p.sum(1, keepdims=True)
        assert np.allclose(got[t], want, atol=1e-5)
        assert np.allclose(lse[t], np.log(p.sum(1)) + s.max(1), atol=1e-5)


def test_workload_generator_is_seeded():
    a = W.Rng(3).normal(1000)
    b = W.Rng(3).normal(1000)
    assert np.array_equal(a, b) and abs(a.mean()) < 0.1 and abs(a.std() - 1) < 0.1
    lay = W.config2_layout(seed=0)
    assert lay.lanes == 64 and 1024 <= lay.context.min() and lay.context.max() < 131072
    used = lay.block_table[lay.block_table > 0]
    assert len(np.unique(used)) == len(used), "pages shared between lanes"
    assert 0 not in used


def test_latent_layout_append_roundtrip(orc):
    """The page-blocked layout written by the oracle's append reads back through latent_rows."""
    rng = W.Rng(8)
    cache = np.zeros((4 * 64, 576), np.uint16)
    rows = W.f32_to_bf16_bits(rng.normal(5 * 576).astype(np.float32)).reshape(5, 576)
    slots = np.array([0, 63, 64, 130, 255], np.int32)
    assert orc.kv_append_bf16(rows, slots, cache) == 0
    assert np.array_equal(W.latent_rows(cache, slots), rows)
    # one block of one page is a contiguous 64 x 64 tile
    page1_block2 = cache.reshape(-1)[64 * 576 + 2 * 64 * 64: 64 * 576 + 3 * 64 * 64].reshape(64, 64)
    assert np.array_equal(page1_block2[0], rows[2, 128:192])
