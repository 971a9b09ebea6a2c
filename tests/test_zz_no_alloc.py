"""hk_moe_grouped_noalloc: the grouped MoE FFN for callers that cannot allocate device memory.

Such callers (an engine that reaches the library only through the C ABI with no CUDA
allocator of its own, a pool allocator that forbids raw cudaMalloc, a step loop that must not
take cudaMalloc's device-wide synchronisation) get an entry point without a workspace argument;
its scratch is a fixed device array inside the library.  This file is collected last so a run
that stops at the first failure has run every other test first; it also passes on its own in a
fresh process.
"""
import numpy as np
import pytest
import torch

import oracle
from hyperkernel_b200 import workload as W

pytestmark = pytest.mark.gpu

TOL = 2e-2  # max-abs-rel, the tolerance of the other FP8 / MoE parity tests


def _problem(hk, cuda, tokens, experts, hidden, inter, top_k, seed):
    inp = W.moe_inputs(tokens, experts, hidden, inter, top_k=top_k, seed=seed)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    x = torch.from_numpy(inp["x"].view(np.int16)).to(cuda).view(torch.bfloat16)
    ids, w = hk.route(dev(inp["logits"]), None, top_k, 1.0)
    offsets, perm_token, _, _ = hk.permute(ids, w, experts)
    xq, sx = hk.quant_fp8(x)
    weights = dict(w13=dev(inp["w13"]), s13=dev(inp["s13"]), w2=dev(inp["w2"]), s2=dev(inp["s2"]))
    # the CPU oracle's expert outputs over the same routed rows (the route, permutation and
    # quantisation are bit-exact against the oracle, so the oracle can take the GPU's copies)
    want = oracle.moe_grouped(xq.cpu().numpy(), sx.cpu().numpy(), offsets.cpu().numpy(),
                              perm_token.cpu().numpy(), hidden, inter, inp["w13"], inp["s13"],
                              inp["w2"], inp["s2"])
    return dict(xq=xq, sx=sx, offsets=offsets, perm_token=perm_token, rows=tokens * top_k,
                hidden=hidden, inter=inter, oracle=want, **weights)


def _call_noalloc(hk, p):
    """Through the C ABI: no workspace pointer or size is passed."""
    rows, hidden = p["rows"], p["hidden"]
    out = torch.empty((rows, hidden), dtype=torch.bfloat16, device=p["xq"].device)
    rc = hk.lib().hk_moe_grouped_noalloc(
        hk.ptr(p["xq"]), hk.ptr(p["sx"]), p["xq"].shape[0], hk.ptr(p["offsets"]),
        hk.ptr(p["perm_token"]), rows, p["offsets"].shape[0] - 1, hidden, p["inter"],
        hk.ptr(p["w13"]), hk.ptr(p["s13"]), hk.ptr(p["w2"]), hk.ptr(p["s2"]), hk.ptr(out),
        hk.stream_ptr())
    hk.check(rc)
    return out


def _f32(a):
    if isinstance(a, torch.Tensor):
        return a.float().cpu().numpy().astype(np.float64)
    return np.asarray(a, np.float64)


def _rel_err(a, b):
    a, b = _f32(a), _f32(b)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def test_noalloc_matches_workspace_entry_point_twice(hk, cuda):
    """Two calls in a row share the one scratch array: the larger problem first, then a smaller
    one that leaves the first call's rows, h and tile list behind in the array.  Each result
    agrees with hk_moe_grouped given a caller workspace and with the CPU oracle."""
    problems = [_problem(hk, cuda, 128, 16, 384, 512, 4, seed=62),
                _problem(hk, cuda, 96, 8, 256, 256, 2, seed=61)]
    for p in problems:
        want = hk.moe_grouped(p["xq"], p["sx"], p["offsets"], p["perm_token"], p["rows"],
                              p["hidden"], p["inter"], p["w13"], p["s13"], p["w2"], p["s2"])
        got = _call_noalloc(hk, p)
        torch.cuda.synchronize()
        assert _rel_err(got, want[: p["rows"]]) <= TOL
        assert _rel_err(got, p["oracle"]) <= TOL
    hk.check_errors()


def test_noalloc_refuses_problems_past_its_scratch(hk, cuda):
    p = _problem(hk, cuda, 8, 4, 128, 128, 2, seed=63)
    out = torch.empty((2048, 128), dtype=torch.bfloat16, device=cuda)
    rc = hk.lib().hk_moe_grouped_noalloc(
        hk.ptr(p["xq"]), hk.ptr(p["sx"]), p["xq"].shape[0], hk.ptr(p["offsets"]),
        hk.ptr(p["perm_token"]), 1025, 4, 128, 128, hk.ptr(p["w13"]), hk.ptr(p["s13"]),
        hk.ptr(p["w2"]), hk.ptr(p["s2"]), hk.ptr(out), hk.stream_ptr())
    assert rc == hk.HK_EINVAL and "at most 1024" in hk.last_error()
    rc = hk.lib().hk_moe_grouped_noalloc(
        hk.ptr(p["xq"]), hk.ptr(p["sx"]), p["xq"].shape[0], hk.ptr(p["offsets"]),
        hk.ptr(p["perm_token"]), 16, 4, 128, 4096, hk.ptr(p["w13"]), hk.ptr(p["s13"]),
        hk.ptr(p["w2"]), hk.ptr(p["s2"]), hk.ptr(out), hk.stream_ptr())
    assert rc == hk.HK_EINVAL and "at most 2048" in hk.last_error()
