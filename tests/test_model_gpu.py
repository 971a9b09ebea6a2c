"""The decode step behind the Kernel boundary: HK_MODEL_MLA through hk_open_mla, driven by the
C++ engine over hk_kernel_ops (admission, prefix cache, block tables, chunked prompts, decode
steps with prompt-lookup drafts verified on the device, logprob replies), against the CPU
restatement of the same decoder (oracle/model.py) with the device's own weights.

Two levels of check:
  * op by op, teacher forced: every entry point the model's forward calls (FP8 projections,
    tcgen05 attention, router, grouped experts + shared expert), fed the oracle's own inputs at
    the model's shapes, is within 2e-2 normwise of the oracle (measured: <= 3e-3), and the
    latent rows the model wrote into its paged cache match the oracle's rows for every position;
  * end to end: each request's emitted tokens are replayed through the oracle (teacher forcing).
    Every projection requantises its input to e4m3 (3 mantissa bits), so two correct
    implementations that differ by one bf16 ulp somewhere drift apart by far more than that at
    the logits: the oracle itself, given its embedding with one ulp of noise on 1% of the
    entries, moves its logprobs by ~0.1-0.2.  The end-to-end bound is therefore that measured
    noise floor (NOISE_FACTOR times the oracle's move under that perturbation, at least 2e-2):
    every (id, logprob) pair the device returned is within it of the oracle's log-softmax, and the
    emitted token is the oracle's greedy choice wherever the oracle's top-2 margin exceeds twice
    the bound.  The router takes every expert (top_k = experts), so no routing decision sits on
    a rounding edge.
"""
import threading

import numpy as np
import pytest

from hyperkernel_b200 import engine as H
from oracle import model as M

pytestmark = pytest.mark.gpu

OP_TOL = 2e-2        # normwise max-abs-rel of each entry point against the oracle
NOISE_FACTOR = 1.5   # end-to-end logprob bound, in units of the oracle's own one-ulp noise floor
PAGE_ROWS, ENTRIES, WIDTH, CHUNK, BLOCK = 64, 8, 4, 64, 3
CONTEXT = PAGE_ROWS * ENTRIES
PAGES = WIDTH * ENTRIES + 9


def _dims(**kw):
    d = dict(hidden=256, q_lora=128, vocab=512, experts=16, top_k=16, inter=128, layers=2, logprobs=4, seed=11,
             rope_theta=10000.0, route_scale=1.0)
    d.update(kw)
    return d


def _device(dims, device=0):
    cfg = H.Config(model=H.MODEL_MLA, page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, width=WIDTH,
                   context=CONTEXT, chunk=CHUNK, block=BLOCK, pages=PAGES, window_pages=PAGES, clip=0,
                   device=device, transport=0)
    return H.Device(cfg, H.MlaModel(**dims))


def _host(ptr, nbytes, dtype):
    from cuda.bindings import runtime as rt

    out = np.empty(nbytes // np.dtype(dtype).itemsize, dtype)
    (err,) = rt.cudaMemcpy(out.ctypes.data, ptr, nbytes, rt.cudaMemcpyKind.cudaMemcpyDeviceToHost)
    assert int(err) == 0, err
    return out


def _weights(dev, d):
    H_, E, I, V, QL = d["hidden"], d["experts"], d["inter"], d["vocab"], d["q_lora"]

    def get(name, dtype, shape, layer=0):
        p, n = dev.tensor(name, layer)
        return _host(p, n, dtype).reshape(shape)

    w = {"embed": get("embed", np.uint16, (V, H_)), "vocab": get("vocab", np.uint8, (V, H_)),
         "vocab.scale": get("vocab.scale", np.float32, (V // 128 if V % 128 == 0 else V // 128 + 1, H_ // 128)),
         "layers": []}
    sc = lambda n, k: ((n + 127) // 128, k // 128)  # noqa: E731
    for layer in range(d["layers"]):
        lw = {}
        for name, n, k in [("wqa", QL, H_), ("wqb", 128 * 576, QL), ("wkva", 576, H_), ("wo", H_, 128 * 512),
                           ("router", E, H_)]:
            lw[name] = get(name, np.uint8, (n, k), layer)
            lw[name + ".scale"] = get(name + ".scale", np.float32, sc(n, k), layer)
        lw["w13"] = get("w13", np.uint8, (E + 1, 2 * I, H_), layer)
        lw["w13.scale"] = get("w13.scale", np.float32, (E + 1,) + sc(2 * I, H_), layer)
        lw["w2"] = get("w2", np.uint8, (E + 1, H_, I), layer)
        lw["w2.scale"] = get("w2.scale", np.float32, (E + 1,) + sc(H_, I), layer)
        w["layers"].append(lw)
    return w


def _requests(vocab, seed):
    """Prompts that cross chunk and page edges, one that repeats a phrase (so prompt lookup
    proposes drafts from the prompt) and two that share a 70-token prefix (the prefix cache)."""
    rng = np.random.default_rng(seed)
    phrase = rng.integers(0, vocab, 9).tolist()
    shared = rng.integers(0, vocab, 70).tolist()
    prompts = [rng.integers(0, vocab, 30).tolist(), rng.integers(0, vocab, 150).tolist(), phrase * 8,
               shared + rng.integers(0, vocab, 5).tolist(), shared + rng.integers(0, vocab, 12).tolist(),
               rng.integers(0, vocab, 1).tolist()]
    return [(p, 14) for p in prompts]


def _run(dev, requests, logprobs):
    eng = H.Engine(H.engine_config(page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, window_keep=0,
                                   context=CONTEXT, width=WIDTH, chunk=CHUNK, block=BLOCK, pad=0, budget=None,
                                   every=1, headroom=2048), dev.ops(), keep=dev)
    samp = H.Sampling(0.0, 1.0, 0, logprobs, 5)
    reqs = [eng.submit(p, lim, sampling=samp) for p, lim in requests]
    eng.close()
    result = {}
    loop = threading.Thread(target=lambda: result.setdefault("rc", eng.run()))
    loop.start()
    loop.join(timeout=600)
    assert not loop.is_alive(), "the engine did not finish"
    assert result["rc"] == 0, eng.failure
    heard = [eng.heard(r) for r in reqs]
    metrics = eng.metrics()
    return heard, metrics


def _noise_floor(w, d, seq, rows):
    """How far the oracle's own logprobs move, at `rows`, when one bf16 ulp of noise lands on 1%
    of the embedding entries: the resolution an FP8 pipeline's logprobs have."""
    rng = np.random.default_rng(len(seq))
    e = w["embed"].copy()
    mask = rng.random(e.shape) < 0.01
    e[mask] ^= 1
    a = M.logits(w, d, seq)
    b = M.logits(dict(w, embed=e), d, seq)
    return max(float(np.abs(M.log_softmax(a[r]) - M.log_softmax(b[r])).max()) for r in rows), a


def _check(w, d, requests, heard):
    checked = exact = 0
    worst = 0.0
    bad = []
    for i, ((prompt, limit), h) in enumerate(zip(requests, heard)):
        assert h.end == "length", (h.end, h.message)
        assert len(h.tokens) == limit
        seq = list(prompt) + list(h.tokens[:-1])
        rows = [len(prompt) - 1 + k for k in range(limit)]
        floor, lg = _noise_floor(w, d, seq, rows)
        bound = max(2e-2, NOISE_FACTOR * floor)
        for k, tok in enumerate(h.tokens):
            p = rows[k]
            row = lg[p]
            top2 = np.sort(row)[-2:]
            lsm = M.log_softmax(row)
            pairs = h.logprobs[k]
            assert pairs and pairs[0][0] == tok, pairs
            err = max(abs(plp - lsm[pid]) for pid, plp in pairs)
            worst = max(worst, err / bound)
            if err > bound:
                bad.append(f"request {i} position {p}: logprob error {err:.3f} > {bound:.3f}")
            if top2[1] - top2[0] > 2 * bound:
                exact += 1
                if tok != int(np.argmax(row)):
                    best = np.argsort(-row)[:4]
                    bad.append(f"request {i} (prompt {len(prompt)}) position {p}: device {tok} "
                               f"(oracle lp {lsm[tok]:.3f}), oracle {int(best[0])}; device pairs "
                               f"{[(a, round(b, 3)) for a, b in pairs]}, oracle top "
                               f"{[(int(b), round(float(lsm[b]), 3)) for b in best]}")
            checked += 1
    assert not bad, f"{len(bad)} mismatches:\n" + "\n".join(bad[:8])
    return checked, exact, worst


def _ops_match_the_oracle(dev, w, d, seq):
    """Each entry point of the forward pass, fed the oracle's own inputs at the model's shapes."""
    import math

    import torch

    from hyperkernel_b200 import _lib as hk
    from hyperkernel_b200 import workload as W
    import oracle

    cuda = torch.device("cuda", 0)
    dv = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    bf = lambda t: W.bf16_bits_to_f32(t.view(torch.int16).cpu().numpy().view(np.uint16))  # noqa: E731

    def rel(a, b):
        return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))

    L, Hd, E, K, I = len(seq), d["hidden"], d["experts"], d["top_k"], d["inter"]
    lw = w["layers"][0]
    errs = {}
    x = M.from_bf16_bits(w["embed"][np.asarray(seq)])
    aq, as_ = M.rms_quant(x)
    for name in ("wqa", "wkva", "router"):
        want = oracle.gemm_fp8(aq, as_, lw[name], lw[name + ".scale"])
        errs[name] = rel(bf(hk.gemm_fp8(dv(aq), dv(as_), dv(lw[name]), dv(lw[name + ".scale"]))), want)
    qa = M.bf16(oracle.gemm_fp8(aq, as_, lw["wqa"], lw["wqa.scale"]))
    qaq, qas = M.rms_quant(qa)
    want = oracle.gemm_fp8(qaq, qas, lw["wqb"], lw["wqb.scale"])
    errs["wqb"] = rel(bf(hk.gemm_fp8(dv(qaq), dv(qas), dv(lw["wqb"]), dv(lw["wqb.scale"]))), want)
    tr = {}
    M.logits(w, d, seq, trace=tr)
    q, kv = tr["q"][0], tr["kv"][0]
    lay = W.paged_layout(W.Rng(1), np.array([0]), np.array([L]), 64)
    cache = np.zeros((lay.num_slots, 576), np.uint16)
    p = oracle.pack(lay.new_rows, lay.context, lay.block_table, 64, lay.num_pages, L)
    oracle.kv_append_bf16(M.bf16_bits(kv), p["slot_mapping"][:L], cache)
    o, _ = hk.mla_decode(dv(M.bf16_bits(q).view(np.int16)).view(torch.bfloat16),
                         dv(cache.view(np.int16)).view(torch.bfloat16), dv(lay.block_table), dv(p["cu_seqlens"]),
                         dv(p["positions"][:L].copy()), 64, L, 1.0 / math.sqrt(576), impl=2)
    errs["attention"] = rel(bf(o), M.attention(q, kv))
    oq, os_ = oracle.quant_fp8(M.bf16_bits(M.bf16(M.attention(q, kv)).reshape(L, -1)))
    want = oracle.gemm_fp8(oq, os_, lw["wo"], lw["wo.scale"])
    errs["wo"] = rel(bf(hk.gemm_fp8(dv(oq), dv(os_), dv(lw["wo"]), dv(lw["wo.scale"]))), want)
    hq, hs = M.rms_quant(M.bf16(x + M.bf16(want)))
    rl = M.bf16(oracle.gemm_fp8(hq, hs, lw["router"], lw["router.scale"]))
    ids, wt = oracle.route(rl, None, K, 1.0)
    gi, gw = hk.route(dv(rl), None, K, 1.0)
    assert np.array_equal(gi.cpu().numpy(), ids)
    off, tok, pw, inv = oracle.permute(ids, wt, E)
    goff, gtok, gpw, ginv = hk.permute(gi, gw, E)
    w13, s13, w2, s2 = lw["w13"], lw["w13.scale"], lw["w2"], lw["w2.scale"]
    yr = oracle.moe_grouped(hq, hs, off, tok, Hd, I, w13[:E], s13[:E], w2[:E], s2[:E])
    gy = hk.moe_grouped(dv(hq), dv(hs), goff, gtok, L * K, Hd, I, dv(w13[:E]), dv(s13[:E]), dv(w2[:E]), dv(s2[:E]))
    errs["experts"] = rel(bf(gy)[:L * K], yr)
    ys = oracle.moe_grouped(hq, hs, np.array([0, L], np.int32), np.arange(L, dtype=np.int32), Hd, I, w13[E:],
                            s13[E:], w2[E:], s2[E:])
    gys = hk.moe_grouped(dv(hq), dv(hs), dv(np.array([0, L], np.int32)), dv(np.arange(L, dtype=np.int32)), L, Hd, I,
                         dv(w13[E:]), dv(s13[E:]), dv(w2[E:]), dv(s2[E:]))
    errs["shared expert"] = rel(bf(gys), ys)
    want = oracle.combine(M.bf16_bits(yr), pw, inv, M.bf16_bits(ys), L, K)
    errs["combine"] = rel(bf(hk.combine(gy, gpw, ginv, gys, L, K)), want)
    hk.check_errors()
    return errs, kv


def test_mla_model_step_through_the_engine_matches_the_oracle(cuda):
    d = _dims()
    dev = _device(d)
    try:
        w = _weights(dev, d)
        requests = _requests(d["vocab"], 3)
        heard, (metrics, accepted, _counts, _sum) = _run(dev, requests, d["logprobs"])
    finally:
        dev.close()
    checked, exact, worst = _check(w, d, requests, heard)
    assert checked == sum(lim for _, lim in requests) and exact >= 5, (exact, checked)
    assert metrics["drafts"] > 0, "no decode step verified drafts"


def test_mla_model_prefill_then_decode_equals_the_whole_sequence(cuda):
    """One lane, block 1 (no drafts), a 130-token prompt over three chunks: every logprob row
    the device returned (the prompt's reply, then each decode step) equals the oracle's row at
    that position."""
    d = _dims(layers=1, experts=16, top_k=16, logprobs=6, seed=5)
    cfg = H.Config(model=H.MODEL_MLA, page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, width=1,
                   context=CONTEXT, chunk=CHUNK, block=1, pages=ENTRIES + 1, window_pages=ENTRIES + 1, clip=0,
                   device=0, transport=0)
    dev = H.Device(cfg, H.MlaModel(**d))
    try:
        w = _weights(dev, d)
        eng = H.Engine(H.engine_config(page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, window_keep=0,
                                       context=CONTEXT, width=1, chunk=CHUNK, block=1, pad=0, budget=None, every=1,
                                       headroom=2048), dev.ops(), keep=dev)
        prompt = np.random.default_rng(8).integers(0, d["vocab"], 130).tolist()
        r = eng.submit(prompt, 20, sampling=H.Sampling(0.0, 1.0, 0, d["logprobs"], 0))
        eng.close()
        assert eng.run() == 0, eng.failure
        h = eng.heard(r)
    finally:
        dev.close()
    checked, exact, worst = _check(w, d, [(prompt, 20)], [h])
    assert checked == 20


def test_mla_model_ops_and_cache_rows_match_the_oracle(cuda):
    """Op by op at the model's shapes (one layer, a 130-token sequence), and the latent rows the
    model wrote into its paged cache while prefilling that sequence over three chunks."""
    d = _dims(layers=1, experts=16, top_k=16, logprobs=2, seed=5)
    cfg = H.Config(model=H.MODEL_MLA, page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, width=1,
                   context=CONTEXT, chunk=CHUNK, block=1, pages=ENTRIES + 1, window_pages=ENTRIES + 1, clip=0,
                   device=0, transport=0)
    dev = H.Device(cfg, H.MlaModel(**d))
    try:
        w = _weights(dev, d)
        eng = H.Engine(H.engine_config(page_rows=PAGE_ROWS, entries=ENTRIES, window=ENTRIES, window_keep=0,
                                       context=CONTEXT, width=1, chunk=CHUNK, block=1, pad=0, budget=None, every=1,
                                       headroom=2048), dev.ops(), keep=dev)
        prompt = np.random.default_rng(8).integers(0, d["vocab"], 130).tolist()
        r = eng.submit(prompt, 2, sampling=H.Sampling(0.0, 1.0, 0, 0, 0))
        eng.close()
        assert eng.run() == 0, eng.failure
        h = eng.heard(r)
        seq = prompt + h.tokens[:1]
        errs, kv = _ops_match_the_oracle(dev, w, d, seq)
        assert max(errs.values()) <= OP_TOL, errs
        # the model's own cache rows: the lane's pages hold its positions in order (pages 1..)
        p, n = dev.tensor("tokens")
        pool = _host(p, n, np.int32).reshape(ENTRIES + 1, PAGE_ROWS)
        p, n = dev.tensor("kv", 0)
        cache = _host(p, n, np.uint16).reshape(ENTRIES + 1, 9, PAGE_ROWS, 64)
        page_of = {}
        for blk in range((len(seq) + PAGE_ROWS - 1) // PAGE_ROWS):
            want_toks = seq[blk * PAGE_ROWS:(blk + 1) * PAGE_ROWS]
            page_of[blk] = next(pg for pg in range(1, ENTRIES + 1) if pool[pg][:len(want_toks)].tolist() == want_toks)
        got = np.stack([M.from_bf16_bits(cache[page_of[t // PAGE_ROWS], :, t % PAGE_ROWS, :].reshape(576))
                        for t in range(len(seq))])
        assert np.abs(got - kv).max() / np.abs(kv).max() <= OP_TOL
    finally:
        dev.close()


def test_mla_model_rejects_bad_configurations(cuda):
    d = _dims()
    for field, value in [("hidden", 200), ("experts", 8), ("vocab", 500), ("top_k", 17)]:
        bad = dict(d, **{field: value})
        with pytest.raises(Exception):
            _device(bad)
    cfg = H.Config(model=H.MODEL_MLA, page_rows=32, entries=ENTRIES, window=ENTRIES, width=WIDTH, context=256,
                   chunk=CHUNK, block=BLOCK, pages=PAGES, window_pages=PAGES, clip=0, device=0, transport=0)
    with pytest.raises(Exception, match="pages of 64"):
        H.Device(cfg, H.MlaModel(**d))
