"""The CPU restatement of the HK_MODEL_MLA decoder (oracle/model.py): its e4m3 encoder against the
C oracle's, and the causal structure the device test relies on (the logits of a prefix are the
first rows of the logits of the whole sequence, so a token's logits depend only on the tokens
before it, however the device batched them)."""
import numpy as np

import oracle
from oracle import model as M


def test_e4m3_encoder_matches_the_c_oracle():
    rng = np.random.default_rng(1)
    x = np.concatenate([rng.standard_normal(4000) * 50, rng.standard_normal(2000) * 0.01,
                        [0.0, -0.0, 448.0, 500.0, -1e9, 2.0 ** -10, 3 * 2.0 ** -10, 240.0, 232.0, 248.0]])
    x = x.astype(np.float32)
    want = np.array([oracle.f32_to_e4m3(float(v)) for v in x], np.uint8)
    got = M.e4m3(x)
    same = got == want
    both_zero = ((got & 0x7F) == 0) & ((want & 0x7F) == 0)  # signed zeros may differ in the sign bit
    assert (same | both_zero).all(), x[~(same | both_zero)][:8]


def _tiny_weights(rng, d):
    H, QL, E, I, V = d["hidden"], d["q_lora"], d["experts"], d["inter"], d["vocab"]

    def q(n, k, count=None):
        shape = (n, k) if count is None else (count, n, k)
        z = rng.standard_normal(shape).astype(np.float32)
        s_shape = ((n + 127) // 128, k // 128) if count is None else (count, (n + 127) // 128, k // 128)
        return M.e4m3(z * 112.0), np.full(s_shape, 1.0 / np.sqrt(k) / 112.0, np.float32)

    w = {"embed": M.bf16_bits(rng.standard_normal((V, H)).astype(np.float32))}
    w["vocab"], w["vocab.scale"] = q(V, H)
    w["layers"] = []
    for _ in range(d["layers"]):
        lw = {}
        for name, n, k in [("wqa", QL, H), ("wqb", 128 * 576, QL), ("wkva", 576, H), ("wo", H, 128 * 512),
                           ("router", E, H)]:
            lw[name], lw[name + ".scale"] = q(n, k)
        lw["w13"], lw["w13.scale"] = q(2 * I, H, E + 1)
        lw["w2"], lw["w2.scale"] = q(H, I, E + 1)
        w["layers"].append(lw)
    return w


def test_oracle_logits_are_causal():
    d = dict(hidden=128, q_lora=128, vocab=256, experts=16, top_k=4, inter=128, layers=1)
    rng = np.random.default_rng(2)
    w = _tiny_weights(rng, d)
    seq = rng.integers(0, d["vocab"], 24)
    whole = M.logits(w, d, seq)
    part = M.logits(w, d, seq[:9])
    assert whole.shape == (24, 256) and np.isfinite(whole).all()
    assert np.array_equal(part, whole[:9])
    assert whole.std() > 0.1
