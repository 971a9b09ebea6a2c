"""The decode step behind the Kernel boundary: HK_MODEL_MLA through hk_open_mla, driven by the
C++ engine over hk_kernel_ops (admission, prefix cache, block tables, chunked prompts, decode
steps with prompt-lookup drafts verified on the device, logprob replies), against the CPU
restatement of the same decoder (oracle/model.py) with the device's own weights.

Each request's emitted tokens are replayed through the oracle with teacher forcing: the token
emitted at position p must be the oracle's greedy choice at p wherever the oracle's top-2 logit
margin exceeds MARGIN (below it, bf16 rounding may legitimately pick the other), and every
(id, logprob) pair the device returned must be within LP_TOL of the oracle's log-softmax.  The
router takes every expert (top_k = experts), so no routing decision sits on a rounding edge.
"""
import ctypes as C
import threading

import numpy as np
import pytest

from hyperkernel_b200 import engine as H
from oracle import model as M

pytestmark = pytest.mark.gpu

MARGIN = 0.05   # logits
LP_TOL = 2e-2   # absolute, on logprobs
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


def _check(w, d, requests, heard):
    checked = exact = 0
    worst = 0.0
    bad = []
    for i, ((prompt, limit), h) in enumerate(zip(requests, heard)):
        assert h.end == "length", (h.end, h.message)
        assert len(h.tokens) == limit
        seq = list(prompt) + list(h.tokens[:-1])
        lg = M.logits(w, d, seq)
        for k, tok in enumerate(h.tokens):
            p = len(prompt) - 1 + k
            row = lg[p]
            top2 = np.sort(row)[-2:]
            lsm = M.log_softmax(row)
            pairs = h.logprobs[k]
            assert pairs and pairs[0][0] == tok, pairs
            err = max(abs(plp - lsm[pid]) for pid, plp in pairs)
            worst = max(worst, err)
            if top2[1] - top2[0] > MARGIN:
                exact += 1
                if tok != int(np.argmax(row)):
                    best = np.argsort(-row)[:4]
                    bad.append(f"request {i} (prompt {len(prompt)}) position {p}: device {tok} "
                               f"(oracle lp {lsm[tok]:.3f}), oracle {int(best[0])}; device pairs "
                               f"{[(a, round(b, 3)) for a, b in pairs]}, oracle top "
                               f"{[(int(b), round(float(lsm[b]), 3)) for b in best]}")
            checked += 1
    assert not bad, f"{len(bad)} of {exact} clear-margin tokens differ:\n" + "\n".join(bad[:8])
    assert worst <= LP_TOL, f"logprob error {worst:.3e}"
    return checked, exact, worst


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
    assert exact >= checked // 2, (exact, checked)
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
    assert checked == 20 and worst <= LP_TOL


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
