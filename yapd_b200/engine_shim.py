"""Drop-in wiring of the select-step library into the reference's engines.

``FlashEngine._step_gpu`` (m8than/yapd ``server/engine.py:491-622``) keeps its
signature; its select body, state update and write-back (``:533-622``) become
one ``select_step`` call.  ``TurboEngine._sample`` (``server/engine_ar.py:220-243``)
keeps its signature and becomes one ``sample_rows`` call.

The engines are duck-typed: any object with the reference's attributes works
(``n_branch, BS, K, temp, tau, cfg, posT, MASK, STOP, V, L, N_max, sched_t,
q_t, log_prior, xt, blk_start, k_step, cache_len, n_speech, is_commit`` for
Flash; ``temp, top_k, top_p, rep_p`` for Turbo).
"""
from __future__ import annotations

import types

import torch

from .select import EngineBuffers, SelectOutputs, sample_rows, select_step


class FlashSelect:
    """State the select step keeps per engine: preallocated outputs and flags,
    and the Philox step counter (the reference draws fresh ``torch.rand``
    noise every tick, ``server/engine.py:88-91``; here every tick advances the
    offset)."""

    def __init__(self, engine, seed: int = 1234):
        self.seed = seed
        self.offset = 0
        self.out = None
        self.flags = None
        self.engine = engine

    def __call__(self, logits: torch.Tensor, B: int, blk_idx: torch.Tensor, xt_blk: torch.Tensor,
                 commit_rows: torch.Tensor):
        """Select body, state update and engine write-back of
        ``FlashEngine._step_gpu`` for rows ``[0, B)`` (``server/engine.py:533-622``):
        one library call (two kernels, no torch op); returns ``(flags, xt_final)``.
        ``k_step``, ``is_commit``, ``xt``, ``cache_len`` and ``blk_start`` are
        updated in the engine's own tensors."""
        e = self.engine
        L = e.BS
        if self.out is None or self.out.xt.shape[0] < B:
            n = max(B, getattr(e, "max_active", B))
            self.out = SelectOutputs.empty(n, L, logits.device)
            self.flags = torch.empty(n, 6, dtype=torch.int64, device=logits.device)
        o = self.out
        out = SelectOutputs(xt=o.xt[:B], sampled=o.sampled[:B], pmi=o.pmi[:B], n_unmask=o.n_unmask[:B],
                            n_mask_after=o.n_mask_after[:B], hit_eos=o.hit_eos[:B],
                            k_step=e.k_step[:B], is_commit=e.is_commit[:B])
        eng = EngineBuffers(xt_full=e.xt, blk_start=e.blk_start[:B], cache_len=e.cache_len[:B],
                            n_speech=e.n_speech[:B], flags=self.flags[:B],
                            blk_limit=int(e.N_max) - L, cache_limit=int(e.L) - L)
        select_step(logits, xt_blk, e.k_step[:B], commit_rows, e.log_prior, e.sched_t, e.q_t,
                    cfg_scale=float(e.cfg) if e.n_branch == 2 else 0.0, mask_id=e.MASK,
                    stop_id=e.STOP, temperature=float(e.temp), pos_noise=e.posT > 0,
                    use_quantile=e.tau > 0, seed=self.seed, offset=self.offset, out=out, engine=eng)
        self.offset += 1
        return self.flags[:B], out.xt


def flash_step_gpu(self, B: int, l_used: int):
    """``FlashEngine._step_gpu`` with the select body on the B200 kernels.

    The forward prelude keeps the engine's own modules (embedding, Llama core,
    speech head); only the select step changed.
    """
    nb = self.n_branch
    blk_idx = self.blk_start[:B, None] + self.ar16
    xt_blk = self.xt[:B].gather(1, blk_idx)
    emb = self.t3._embed_speech_tokens(xt_blk).to(self.dtype)
    x = emb.repeat_interleave(nb, dim=0) if nb == 2 else emb
    pos1 = self.cache_len[:B, None] + self.ar16
    pos = pos1.repeat_interleave(nb, dim=0) if nb == 2 else pos1
    colv1 = torch.where(self.arL[None, :l_used] < (self.cache_len[:B, None] + self.BS), 0.0,
                        float("-inf"))
    colv = colv1.repeat_interleave(nb, dim=0) if nb == 2 else colv1
    mask = colv[:, None, None, :].to(self.dtype)
    hidden = self.core.forward(x, pos, pos, self.kc, self.vc, mask, self_attn_only=False, l_used=l_used)
    shift_hidden = torch.cat([self.shift_ctx[:B * nb], hidden[:, : self.BS - 1]], dim=1)
    logits = self.t3.speech_head(shift_hidden)
    commit_rows = self.is_commit[:B].clone()
    last_h = hidden[:, self.BS - 1: self.BS]
    cm2 = commit_rows.repeat_interleave(nb) if nb == 2 else commit_rows
    self.shift_ctx[:B * nb] = torch.where(cm2[:, None, None], last_h, self.shift_ctx[:B * nb])
    if logits.dtype not in (torch.float32, torch.bfloat16):
        logits = logits.float()
    return self._yapd_select(logits, B, blk_idx, xt_blk, commit_rows)


def install_flash(engine, seed: int = 1234):
    """Route ``engine._step_gpu`` through the B200 select step."""
    engine._yapd_select = FlashSelect(engine, seed)
    engine._step_gpu = types.MethodType(flash_step_gpu, engine)
    return engine


def turbo_sample(self, logits: torch.Tensor, seen: torch.Tensor) -> torch.Tensor:
    """``TurboEngine._sample`` (temperature -> top-k -> top-p -> repetition
    penalty -> Gumbel-max) on the B200 kernel; returns ``(B,)`` int64 ids."""
    st = getattr(self, "_yapd_turbo_offset", 0)
    self._yapd_turbo_offset = st + 1
    out = sample_rows(logits, temperature=float(self.temp), top_k=int(self.top_k),
                      top_p=float(self.top_p), rep_penalty=float(self.rep_p), seen=seen,
                      seed=getattr(self, "_yapd_seed", 4321), offset=st, zero_temp_greedy=False)
    return out.long()


def install_turbo(engine, seed: int = 4321):
    """Route ``engine._sample`` through the B200 sampling kernel."""
    engine._yapd_seed = seed
    engine._sample = types.MethodType(turbo_sample, engine)
    return engine
