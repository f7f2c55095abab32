"""CPU oracle for the block-diffusion select step (test infrastructure only).

This module is the checker for the CUDA path, never the product: only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` import it.

It restates, with torch CPU operators in the reference's own order, the
select body of Chatterbox-Flash's continuous-batching engine
(``server/engine.py:533-593`` of m8than/yapd) and the sampling chain of its
Turbo engine (``server/engine_ar.py:220-243``).  Float results depend on the
order of operations, so each formula keeps the reference's op sequence:

* CFG: ``guided = lsc + w*(lsc - lsu)`` on log-softmaxes (``engine.py:536-538``);
* probabilities ``softmax(c)``, ``softmax(u)`` (``engine.py:539-540``);
* token choice ``argmax(guided / T + G)`` (``engine.py:546-550``);
* filters: ``/T`` -> top-k (sorted) -> top-p keep iff ``cumsum - p < top_p``
  -> repetition penalty ``v>0 ? v/r : v*r`` -> ``+G`` -> argmax over the
  sorted candidates (``engine_ar.py:230-243``);
* PMI ``log(max(p,1e-8)) - lambda*log_prior`` and the CFG combination
  ``(1+w)*pmi_c - w*pmi_u`` (``engine.py:553-558``, ``calibration.py:56-60``,
  ``cfg_guidance.py:50-57``);
* position noise, quantile threshold, count schedule and rank-based unmask
  (``engine.py:559-593``).

Deterministic tie rules, where the reference's sorts are unstable
(``torch.topk``, ``argsort``): equal values keep ascending index order.  On
inputs without exact ties the oracle equals the unmodified reference; the
fixtures under ``tests/golden`` were produced by the reference itself.

Extensions beyond the reference (parity-unpinned against upstream, reducing
to the reference when disabled): min-p (keep iff ``p >= min_p * p_max`` over
the same top-k softmax the top-p filter uses, applied after top-p), per-request
filter parameters, ``pmi_lambda != 1``.

Torch version drift: the reference pins torch 2.7.1 (``uv.lock``); this oracle
runs on the image's torch.  The fixtures record the version that made them.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import philox

NEG_INF = float("-inf")


def gumbel_from_uniform(u: torch.Tensor) -> torch.Tensor:
    """``-log(max(-log(max(u,1e-20)),1e-20))`` (``server/engine.py:88-91``)."""
    u = u.clamp_min(1e-20)
    return -torch.log((-torch.log(u)).clamp_min(1e-20))


def philox_noise(seed: int, offset: int, B: int, L: int, V: int):
    """Token noise ``(B, L, V)`` and position noise ``(B, L)`` of the kernels'
    in-kernel generator (counter layout in ``oracle/philox.py``)."""
    gt = gumbel_from_uniform(philox.token_uniforms(seed, offset, B, L, V))
    gp = gumbel_from_uniform(philox.position_uniforms(seed, offset, B, L))
    return gt, gp


def philox_noise_rows(seed: int, offset: int, rows, L: int, V: int):
    """Token noise ``(n, L, V)`` and position noise ``(n, L)`` of requests
    ``rows`` (original indices) of a batch with block length ``L``."""
    import numpy as np
    flat = (np.asarray(rows, dtype=np.int64)[:, None] * L + np.arange(L)[None, :]).reshape(-1)
    gt = gumbel_from_uniform(philox.token_uniforms_at(seed, offset, flat, V)).view(len(rows), L, V)
    gp = gumbel_from_uniform(philox.position_uniforms_at(seed, offset, flat)).view(len(rows), L)
    return gt, gp


def cfg_combine(logits: torch.Tensor, nb: int, L: int, w: float):
    """``server/engine.py:533-544``: returns ``guided, probs_c, probs_u``
    each ``(B, L, V)`` (``probs_u`` is None without CFG)."""
    logits = logits.float()
    V = logits.shape[-1]
    B = logits.shape[0] // nb
    if nb == 2:
        lc = logits.view(B, 2, L, V)
        logits_c, logits_u = lc[:, 0], lc[:, 1]
        lsc = F.log_softmax(logits_c, dim=-1)
        lsu = F.log_softmax(logits_u, dim=-1)
        guided = lsc + w * (lsc - lsu)
        probs_c = logits_c.softmax(-1)
        probs_u = logits_u.softmax(-1)
    else:
        guided = logits
        probs_c = logits.softmax(-1)
        probs_u = None
    return guided, probs_c, probs_u


def is_filtered(V: int, top_k, top_p, min_p, rep, has_history: bool) -> torch.Tensor:
    """Rows that go through the filter chain (``engine_ar.py:230-241``) rather
    than the plain ``argmax(guided/T + G)`` of ``engine.py:546-550``."""
    f = ((top_k > 0) & (top_k < V)) | (top_p < 1.0) | (min_p > 0.0)
    if has_history:
        f = f | (rep != 1.0)
    return f


def sample_tokens(guided: torch.Tensor, T, top_k, top_p, min_p, rep, seen, G,
                  zero_temp: str = "greedy") -> torch.Tensor:
    """Sampled token per row of ``guided`` ``(R, V)``.

    ``T, top_k, top_p, min_p, rep``: per-row ``(R,)`` tensors.  ``seen``:
    ``(R, V)`` bool history or None.  ``G``: ``(R, V)`` Gumbel noise indexed by
    vocabulary id.  ``zero_temp``: ``"greedy"`` (``T <= 0`` takes the argmax
    with no noise, ``engine.py:549-550``) or ``"unscaled"`` (``T <= 0`` skips the
    division but still samples, ``engine_ar.py:230-231``).
    """
    R, V = guided.shape
    out = torch.empty(R, dtype=torch.long)
    filt = is_filtered(V, top_k, top_p, min_p, rep, seen is not None)
    noisy = (T > 0) | (zero_temp == "unscaled")
    # ---- unfiltered rows: engine.py:546-550 ----
    for t_pos in (True, False):
        rows = (~filt) & ((T > 0) == t_pos)
        if not bool(rows.any()):
            continue
        g = guided[rows]
        if t_pos:
            score = g / T[rows][:, None] + G[rows]
        elif zero_temp == "unscaled":
            score = g + G[rows]
        else:
            score = g
        out[rows] = score.argmax(-1)
    # ---- filtered rows: engine_ar.py:230-243 (grouped by k) ----
    if bool(filt.any()):
        k_eff = torch.where((top_k > 0) & (top_k < V), top_k.long(), torch.full_like(top_k.long(), V))
        for kval in sorted(set(k_eff[filt].tolist())):
            rows = filt & (k_eff == kval)
            x = guided[rows]
            t = T[rows]
            scale = (t > 0) & (t != 1.0)
            x = torch.where(scale[:, None], x / torch.where(scale, t, torch.ones_like(t))[:, None], x)
            vals, idx = torch.sort(x, dim=-1, descending=True, stable=True)
            vals, idx = vals[:, :kval], idx[:, :kval]
            tp = top_p[rows]
            mp = min_p[rows]
            if bool(((tp < 1.0) | (mp > 0.0)).any()):
                probs = vals.softmax(-1)
                cum_before = probs.cumsum(-1) - probs
                drop_p = (tp < 1.0)[:, None] & ~(cum_before < tp[:, None])
                drop_m = (mp > 0.0)[:, None] & ~(probs >= mp[:, None] * probs[:, :1])
                vals = torch.where(drop_p | drop_m, torch.full_like(vals, NEG_INF), vals)
            rp = rep[rows]
            if seen is not None:
                seen_k = seen[rows].gather(1, idx)
                pen = torch.where(vals > 0, vals / rp[:, None], vals * rp[:, None])
                vals = torch.where(seen_k & (rp != 1.0)[:, None], pen, vals)
            nz = noisy[rows]
            score = torch.where(nz[:, None], vals + G[rows].gather(1, idx), vals)
            choice = score.argmax(-1, keepdim=True)
            out[rows] = idx.gather(1, choice).squeeze(1)
    return out


def pmi_scores(sampled, probs_c, probs_u, log_prior, w: float, lam: float):
    """``server/engine.py:553-558`` with ``calibration.py:58-60``'s lambda."""
    s = sampled.unsqueeze(-1)
    lp = log_prior[sampled]
    lpl = lp if lam == 1.0 else lam * lp
    lp_c = probs_c.gather(-1, s).squeeze(-1).clamp_min(1e-8).log()
    pmi = lp_c - lpl
    if probs_u is not None:
        lp_u = probs_u.gather(-1, s).squeeze(-1).clamp_min(1e-8).log()
        pmi_u = lp_u - lpl
        pmi = (1.0 + w) * pmi - w * pmi_u
    return pmi


def unmask_select(pmi, xt, sampled, k_step, is_commit, sched_t, q_t, *, mask_id: int,
                  stop_id: int, num_steps: int, use_quantile: bool):
    """``server/engine.py:563-593``; argsort made stable (lower position first)."""
    B, L = xt.shape
    K = num_steps
    is_mask = xt == mask_id
    m = is_mask.sum(1)
    ks = k_step
    kc = ks.clamp(max=K - 1)
    asc = torch.where(is_mask, pmi, torch.inf).sort(1).values
    p = q_t[kc] * (m - 1).clamp_min(0).float()
    lo = p.floor().long().clamp_min(0)
    hi = p.ceil().long().clamp_min(0)
    v_lo = asc.gather(1, lo[:, None]).squeeze(1)
    v_hi = asc.gather(1, hi[:, None]).squeeze(1)
    tau_k = v_lo + (p - lo.float()) * (v_hi - v_lo)
    n_quant = ((pmi >= tau_k[:, None]) & is_mask).sum(1)
    if not use_quantile:
        n_quant = torch.zeros_like(n_quant)
    n_sched = torch.minimum(sched_t[kc], m)
    n_unmask = torch.minimum(torch.maximum(n_sched, n_quant), m)
    n_unmask = torch.where(ks >= K - 1, m, n_unmask)
    n_unmask = torch.where(m == 0, torch.zeros_like(n_unmask), n_unmask)
    order = torch.argsort(torch.where(is_mask, pmi, -torch.inf), dim=1, descending=True, stable=True)
    rank = torch.empty_like(order)
    rank.scatter_(1, order, torch.arange(L).expand(B, -1).contiguous())
    do_unmask = is_mask & (rank < n_unmask[:, None])
    xt_new = torch.where(do_unmask, sampled, xt)
    denoise = ~is_commit
    xt_final = torch.where(denoise[:, None], xt_new, xt)
    n_mask_after = (xt_final == mask_id).sum(1)
    hit_eos = (xt_final == stop_id).any(1)
    k_step_new = torch.where(denoise, ks + 1, ks)
    # commit-phase transitions, engine.py:595-612 (cache/block offsets are the caller's)
    commit = is_commit
    k_step_final = torch.where(commit, torch.zeros_like(ks), k_step_new)
    to_commit = denoise & ~hit_eos & ((n_mask_after == 0) | (k_step_final >= K))
    is_commit_final = torch.where(commit, torch.zeros_like(commit), commit) | to_commit
    return dict(xt_final=xt_final, n_unmask=n_unmask, do_unmask=do_unmask & denoise[:, None],
                n_mask_after=n_mask_after, hit_eos=hit_eos, k_step=k_step_new, tau=tau_k,
                k_step_final=k_step_final, is_commit_final=is_commit_final)


def select_step(inp, *, noise: str = "explicit", seed: int = 0, offset: int = 0,
                zero_temp: str = "greedy", per_row_params: bool = True) -> dict:
    """Whole step for a ``yapd_b200.workloads.StepInputs``-like object.

    Returns ``sampled (B,L)``, ``pmi (B,L)`` (after position noise),
    ``xt_final``, ``n_unmask``, ``n_mask_after``, ``hit_eos``, ``k_step`` and
    ``filtered (B,)``.  ``noise``: ``"explicit"`` uses ``inp.gumbel_tok`` /
    ``inp.gumbel_pos``; ``"philox"`` regenerates the kernels' noise.
    """
    B, L, V = inp.B, inp.L, inp.V
    guided, probs_c, probs_u = cfg_combine(inp.logits, inp.nb, L, inp.cfg_scale)
    if noise == "explicit":
        gt, gp = inp.gumbel_tok, inp.gumbel_pos
    else:
        gt, gp = philox_noise(seed, offset, B, L, V)
    rep_rows = lambda x: x.repeat_interleave(L)
    seen = None if inp.history is None else inp.history.repeat_interleave(L, dim=0)
    sampled = sample_tokens(
        guided.reshape(B * L, V), rep_rows(inp.temperature), rep_rows(inp.top_k),
        rep_rows(inp.top_p), rep_rows(inp.min_p), rep_rows(inp.rep_penalty), seen,
        gt.reshape(B * L, V), zero_temp=zero_temp).view(B, L)
    pmi = pmi_scores(sampled, probs_c, probs_u, inp.log_prior, inp.cfg_scale, inp.pmi_lambda)
    is_mask = inp.xt == inp.mask_id
    if inp.pos_noise:
        pmi = torch.where(is_mask, pmi + gp, pmi)
    res = unmask_select(pmi, inp.xt, sampled, inp.k_step, inp.is_commit, inp.sched_t, inp.q_t,
                        mask_id=inp.mask_id, stop_id=inp.stop_id, num_steps=inp.num_steps,
                        use_quantile=inp.use_quantile)
    res.update(sampled=sampled, pmi=pmi,
               filtered=is_filtered(V, inp.top_k, inp.top_p, inp.min_p, inp.rep_penalty,
                                    inp.history is not None))
    return res

def engine_update(res, xt_full, blk_start, cache_len, n_speech, is_commit, *, L: int,
                  blk_limit: int, cache_limit: int):
    """The engine-side write-back of ``server/engine.py:586-622`` after
    ``unmask_select``: scatter ``xt_final`` into the token buffer at
    ``blk_start``, advance the cache length and block start of the rows that
    were committing (clamped), and pack the flags ``(B, 6)``.  Returns
    ``(xt_full, blk_start, cache_len, flags)`` (new tensors)."""
    B = blk_start.shape[0]
    ar = torch.arange(L)
    blk_idx = blk_start[:, None] + ar
    xt_full = xt_full.clone()
    xt_full[:B] = xt_full[:B].scatter(1, blk_idx, res["xt_final"])
    adv = is_commit
    cache_len = torch.where(adv, (cache_len + L).clamp(max=cache_limit), cache_len)
    blk_start = torch.where(adv, (blk_start + L).clamp(max=blk_limit), blk_start)
    flags = torch.stack([adv.long(), res["n_mask_after"].long(), res["hit_eos"].long(),
                         res["k_step_final"].long(), blk_start, n_speech.long()], dim=1)
    return xt_full, blk_start, cache_len, flags


def offline_gumbel(u: torch.Tensor) -> torch.Tensor:
    """The offline generator's Gumbel transform ``-log(-log(u + 1e-10) + 1e-10)``
    (``chatterbox_flash/model.py:76-80``)."""
    return -torch.log(-torch.log(u + 1e-10) + 1e-10)


def offline_block_step(logits_cond, logits_uncond, xt, done, *, k: int, K: int, sched_k: int,
                       time_shift_tau: float, prior, cfg_scale: float, temperature: float,
                       position_temperature: float, G, Gpos, mask_id: int, stop_id: int):
    """Every row of one step of ``ChatterboxFlashT3.generate``'s block loop
    (``chatterbox_flash/model.py:856-906``): ``_pmi_count_early_step_unmask``
    (``model.py:185-311``) per row not yet done, with ``temperature_sampling=
    "gumbel"`` and explicit noise (``G`` ``(B, bl, V)``, ``Gpos`` ``(B, bl)``),
    the prior override path, then the row's done flag.  Returns ``(xt, done)``."""
    B, bl = xt.shape
    xt = xt.clone()
    done = done.clone()
    for b in range(B):
        if bool(done[b]):
            continue
        c = logits_cond[b].float()
        if cfg_scale != 0.0 and logits_uncond is not None:
            u = logits_uncond[b].float()
            guided = F.log_softmax(c, dim=-1)
            guided = guided + cfg_scale * (guided - F.log_softmax(u, dim=-1))
            pc, pu = F.softmax(c, dim=-1), F.softmax(u, dim=-1)
        else:
            guided, pc, pu = c, F.softmax(c, dim=-1), None
        if temperature > 0:
            sampled = (guided / temperature + G[b]).argmax(-1)
        else:
            sampled = guided.argmax(-1)
        is_mask = xt[b] == mask_id
        s1 = sampled.unsqueeze(1)
        lp = prior[sampled].clamp_min(1e-8).log()
        pmi = pc.gather(1, s1).squeeze(1).clamp_min(1e-8).log() - 1.0 * lp
        if pu is not None:
            pmi_u = pu.gather(1, s1).squeeze(1).clamp_min(1e-8).log() - 1.0 * lp
            pmi = (1.0 + cfg_scale) * pmi - cfg_scale * pmi_u
        if position_temperature > 0:
            pmi = torch.where(is_mask, pmi + (torch.zeros_like(pmi) / position_temperature + Gpos[b]), pmi)
        if k == K - 1:
            do_unmask = is_mask
        else:
            idx = torch.arange(bl)[is_mask]
            m = int(idx.numel())
            do_unmask = torch.zeros_like(is_mask)
            if m > 0:
                pm = pmi[idx]
                n_sched = max(0, min(int(sched_k), m))
                if time_shift_tau > 0:
                    q = max(0.0, 1.0 - time_shift_tau * (k + 1) / K)
                    tau_k = torch.quantile(pm.float(), q)
                    n_quant = int((pm >= tau_k).sum())
                else:
                    n_quant = 0
                n_un = min(max(n_sched, n_quant), m)
                if n_un >= m:
                    do_unmask[idx] = True
                elif n_un > 0:
                    order = torch.argsort(pm, descending=True, stable=True)[:n_un]
                    do_unmask[idx[order]] = True
        xt[b] = torch.where(do_unmask, sampled, xt[b])
        if int((xt[b] == mask_id).sum()) == 0 or bool((xt[b] == stop_id).any()):
            done[b] = True
    return xt, done
