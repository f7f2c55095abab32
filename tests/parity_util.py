"""Helpers for GPU-vs-oracle parity checks.

Sampled ids and committed masks must match the oracle exactly.  The only
tolerated difference is a *certified near-tie*: a position where recomputing
the decision in float64 shows the two candidates within a few float32 ulps of
each other (argmax near-tie, a top-p / min-p / top-k boundary, or a PMI tie at
the unmask cut), so that the float32 rounding of torch CPU and of the kernel
legitimately decide differently.  Tests assert zero uncertified mismatches and
report the certified count.
"""
from __future__ import annotations

import math
import os

import numpy as np
import torch

from oracle import select_oracle as O

PMI_RTOL = 1e-5
# A certified near-tie is a decision whose two sides, recomputed in float64,
# lie within TIE_ULPS units in the last place of float32 at their magnitude.
# Where the kernel and torch CPU can differ: the row sums behind the log-softmax
# and the top-p probabilities are added in different orders (8194 float32 terms:
# the two sums differ by a few ulps), logs and exponentials are rounded by
# different libraries (1-2 ulps each), and a value passes through at most four
# such roundings before a comparison.  16 ulps covers that with a factor of two;
# measured gaps of the certified cases are reported by every test.
TIE_ULPS = 16
# every certified case of the session: (test, b, l, kind, gap in ulps)
CERTIFIED: list = []


def ulp32(x: float) -> float:
    """Spacing of float32 numbers at magnitude |x| (the smallest normal spacing below 2^-126)."""
    x = abs(float(x))
    if x < 2.0 ** -126:
        return 2.0 ** -149
    return 2.0 ** (math.floor(math.log2(x)) - 23)


def gap_ulps(a: float, b: float) -> float:
    """|a - b| in float32 ulps at the larger magnitude."""
    return abs(float(a) - float(b)) / ulp32(max(abs(float(a)), abs(float(b))))


def run_gpu(inp, *, noise="explicit", seed=0, offset=0, dense=True, zero_temp_greedy=True,
            history_as="bitmap", scalar_minp=False):
    """One select step on the GPU.  ``scalar_minp``: pass min-p as the scalar 0
    (every request has it off), which launches the grouped kernel alone for
    bf16 select steps instead of the warp kernel."""
    from yapd_b200 import select as S
    dev = torch.device("cuda")
    hist = None
    if inp.history is not None:
        hist = inp.history_bitmap() if history_as == "bitmap" else inp.history
    if scalar_minp:
        assert float(inp.min_p.max()) <= 0.0
        min_p = 0.0
    else:
        min_p = inp.min_p.to(dev)
    kw = {}
    if noise == "explicit":
        kw = dict(gumbel_tok=inp.gumbel_tok.to(dev), gumbel_pos=inp.gumbel_pos.to(dev))
    out = S.select_step(
        inp.logits.to(dev), inp.xt.to(dev), inp.k_step.to(dev), inp.is_commit.to(dev),
        inp.log_prior.to(dev), inp.sched_t.to(dev), inp.q_t.to(dev), cfg_scale=inp.cfg_scale,
        mask_id=inp.mask_id, stop_id=inp.stop_id, temperature=inp.temperature.to(dev),
        top_k=inp.top_k.to(dev), top_p=inp.top_p.to(dev), min_p=min_p,
        rep_penalty=inp.rep_penalty.to(dev), history=None if hist is None else hist.to(dev),
        pmi_lambda=inp.pmi_lambda, pos_noise=inp.pos_noise, use_quantile=inp.use_quantile,
        seed=seed, offset=offset, zero_temp_greedy=zero_temp_greedy, dense=dense, **kw)
    torch.cuda.synchronize()
    return {k: getattr(out, k).cpu() for k in
            ("xt", "sampled", "pmi", "n_unmask", "n_mask_after", "hit_eos", "k_step", "is_commit")}


def _f64_rows(inp, b, l):
    """float64 guided values of position (b, l)."""
    x = inp.logits.double()
    B, L, V = inp.B, inp.L, inp.V
    if inp.nb == 2:
        lc = x.view(B, 2, L, V)
        c, u = lc[b, 0, l], lc[b, 1, l]
        lsc = torch.log_softmax(c, -1)
        lsu = torch.log_softmax(u, -1)
        g = lsc + inp.cfg_scale * (lsc - lsu)
    else:
        g = x[b, l]
    return g


def certify_token(inp, b, l, a, o, G):
    """(certified, kind, gap in ulps) for tokens a (GPU) and o (oracle) at
    (b, l): certified when a float64 recomputation puts the deciding
    quantities within TIE_ULPS float32 ulps (a score tie, or one of the two
    tokens on a top-k / top-p / min-p boundary)."""
    g = _f64_rows(inp, b, l)
    V = inp.V
    T = float(inp.temperature[b])
    vals = g / T if T > 0 else g.clone()
    top_k, top_p = int(inp.top_k[b]), float(inp.top_p[b])
    min_p, rep = float(inp.min_p[b]), float(inp.rep_penalty[b])
    filt = bool(O.is_filtered(V, inp.top_k[b:b + 1], inp.top_p[b:b + 1], inp.min_p[b:b + 1],
                              inp.rep_penalty[b:b + 1], inp.history is not None)[0])
    Gd = G.double()
    if not filt:
        gp = gap_ulps(vals[a] + Gd[a], vals[o] + Gd[o])
        return gp <= TIE_ULPS, "score", gp
    order = torch.argsort(vals, descending=True, stable=True)
    k = top_k if 0 < top_k < V else V
    vs = vals[order[:k]]
    p = torch.softmax(vs, -1)
    cb = torch.cumsum(p, -1) - p
    rank = torch.empty(V, dtype=torch.long)
    rank[order] = torch.arange(V)

    # the top-p cut: ranks [0, R) kept (cumsum - p < top_p)
    R = int((cb < top_p).sum()) if top_p < 1 else k

    def across(t, cut):
        """Gap between token t and the value on the other side of a cut at
        rank `cut` (ranks [0, cut) kept): a token whose value is that close to
        the last kept / first dropped value can fall on either side when the
        two implementations round their values a few ulps apart."""
        r = int(rank[t])
        if r < cut:
            return gap_ulps(vals[t], vs[cut]) if cut < vs.numel() else float("inf")
        return gap_ulps(vals[t], vs[cut - 1]) if cut > 0 else float("inf")

    def boundary(t):
        """(kind, gap) of the nearest filter boundary of token t."""
        r = int(rank[t])
        best = ("none", float("inf"))
        cands = []
        if 0 < top_k < V:
            cands.append(("top-k", gap_ulps(vals[t], vals[order[k]]) if r < k else gap_ulps(vals[t], vs[-1])))
        if top_p < 1:
            if r < k:
                cands.append(("top-p", gap_ulps(cb[r], top_p)))
            cands.append(("top-p-order", across(t, R)))
        if r < k and min_p > 0:
            cands.append(("min-p", gap_ulps(p[r] / p[0], min_p)))
        for c in cands:
            if c[1] < best[1]:
                best = c
        return best

    ba, bo = boundary(a), boundary(o)
    bnd = ba if ba[1] <= bo[1] else bo
    if bnd[1] <= TIE_ULPS:
        return True, bnd[0], bnd[1]

    def score(t):
        v = vals[t]
        if inp.history is not None and rep != 1.0 and bool(inp.history[b, t]):
            v = v / rep if v > 0 else v * rep
        return v + Gd[t]
    gp = gap_ulps(score(a), score(o))
    return gp <= TIE_ULPS, "score", gp


def compare(inp, gpu, orc, G, positions=None, report=None):
    """Assert parity of sampled / pmi / xt / counters; returns counts."""
    B, L = inp.B, inp.L
    s_g, s_o = gpu["sampled"].long(), orc["sampled"]
    if positions is None:
        positions = torch.ones(B, L, dtype=torch.bool)
    mism = (s_g != s_o) & positions
    certified = 0
    bad_rows = set()
    test = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    for b, l in mism.nonzero().tolist():
        a, o = int(s_g[b, l]), int(s_o[b, l])
        ok, kind, gp = (False, "range", float("inf")) if (a < 0 or a >= inp.V) else \
            certify_token(inp, b, l, a, o, G[b, l])
        if not ok:
            raise AssertionError(f"sampled mismatch at ({b},{l}): gpu {a} oracle {o} "
                                 f"(nearest tie: {kind}, {gp:.1f} ulps)")
        certified += 1
        CERTIFIED.append((test, b, l, kind, gp))
        bad_rows.add(b)
    # PMI where the same token was sampled
    same = positions & ~mism
    pg, po = gpu["pmi"][same].double(), orc["pmi"][same].double()
    err = (pg - po).abs() / po.abs().clamp_min(1.0)
    if err.numel():
        worst = float(err.max())
        assert worst <= PMI_RTOL, f"pmi rel err {worst:.3g} > {PMI_RTOL}"
    # committed masks / xt_final: exact except in rows with a certified difference
    pm = orc["pmi"]
    for b in range(B):
        if b in bad_rows:
            continue
        if not torch.equal(gpu["xt"][b], orc["xt_final"][b]):
            # allow a PMI near-tie at the rank cut
            # a PMI near-tie at the rank cut: two masked positions whose PMI the
            # kernel and the oracle each get within PMI_RTOL of the truth
            is_mask = inp.xt[b] == inp.mask_id
            v = pm[b][is_mask].double().sort(descending=True).values
            gaps = (v[:-1] - v[1:]).abs() if v.numel() > 1 else torch.tensor([1.0])
            rel = float(gaps.min()) / max(1.0, float(v.abs().max()))
            if rel <= 2 * PMI_RTOL:
                certified += 1
                CERTIFIED.append((test, b, -1, "pmi-rank", rel / PMI_RTOL))
                continue
            raise AssertionError(f"xt_final mismatch in row {b}: gpu {gpu['xt'][b].tolist()} "
                                 f"oracle {orc['xt_final'][b].tolist()}")
        assert int(gpu["n_mask_after"][b]) == int(orc["n_mask_after"][b])
        assert bool(gpu["hit_eos"][b]) == bool(orc["hit_eos"][b])
        assert int(gpu["k_step"][b]) == int(orc["k_step_final"][b])
        assert bool(gpu["is_commit"][b]) == bool(orc["is_commit_final"][b])
    if report is not None:
        report["certified"] = report.get("certified", 0) + certified
    return certified
