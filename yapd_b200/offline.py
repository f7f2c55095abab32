"""One diffusion step of every row of the offline block generator, in one call.

The reference's offline generator ``ChatterboxFlashT3.generate`` (m8than/yapd
``chatterbox_flash/model.py:856-912``) walks each block's diffusion steps and,
inside every step, loops over the batch rows calling
``_pmi_count_early_step_unmask`` (``model.py:185-311``) once per row, with
host syncs at ``model.py:295``, ``:306`` and ``:898``.  ``block_step`` does that
step for all rows at once on the select-step kernels (two launches, no host
sync): CFG-guided sampling, prior-calibrated PMI against the precomputed
unconditional prior (``prior_override_v``), position noise, the count
schedule / quantile unmask rule with ``torch.quantile``'s interpolation, and
the block-done flags (``model.py:896-906``).

Differences from the reference, by design:

* ``temperature_sampling="multinomial"`` (the reference's default,
  ``model.py:534``) draws with ``torch.multinomial`` from ``softmax(guided/T)``;
  the kernels draw the same distribution by Gumbel-max with their own Philox
  noise, so the samples are equal in distribution, not bit for bit.  With
  ``temperature_sampling="gumbel"`` and the reference's noise passed in
  (``gumbel_tok``, ``gumbel_pos``: ``-log(-log(u + 1e-10) + 1e-10)`` of the
  uniforms ``model.py:76-80`` draws) the outputs are the reference's.
* Only the ``prior_override_v`` path (``pmi_uncond_prior_precompute=True``,
  the generator's default) is covered; the per-block marginal fallback needs
  every position's probabilities at every sampled token.
"""
from __future__ import annotations

import torch

from .select import SelectOutputs, select_step


def block_step(blk_logits: torch.Tensor, xt_blk: torch.Tensor, done: torch.Tensor, k: int, *,
               cfg_scale: float, temperature: float, log_prior: torch.Tensor, sched_t: torch.Tensor,
               q_t: torch.Tensor, mask_id: int, stop_id: int, position_noise: bool = True,
               use_quantile: bool = True, gumbel_tok: torch.Tensor | None = None,
               gumbel_pos: torch.Tensor | None = None, seed: int = 0, offset: int = 0,
               out: SelectOutputs | None = None):
    """Step ``k`` of the current block for every row.

    ``blk_logits``: the block's speech-head logits as the generator holds them,
    ``(2*B, bl, V)`` with the conditional rows first and the unconditional rows
    after them when ``cfg_scale > 0`` (``model.py:862-868``), else ``(B, bl, V)``.
    ``xt_blk``: ``(B, bl)`` int64 block tokens (``xt[:B, bs:be]``).  ``done``:
    ``(B,)`` bool rows whose block already finished (they are left alone).
    ``log_prior``: ``log(clamp(prior_override_v, 1e-8))``; ``sched_t`` the
    OmniVoice count schedule, ``q_t`` the shifted quantiles
    ``max(0, 1 - tau*(k+1)/K)``.  Returns ``(xt_new, done_new)``.
    """
    B, bl = xt_blk.shape
    V = blk_logits.shape[-1]
    dev = blk_logits.device
    if cfg_scale > 0:
        if blk_logits.shape[0] < 2 * B:
            raise ValueError("with CFG, blk_logits holds B conditional then B unconditional rows")
        # (B, 2, bl, V) view: request b, branch 0 = row b, branch 1 = row B + b
        logits = blk_logits[: 2 * B].view(2, B, bl, V).transpose(0, 1)
    else:
        logits = blk_logits[:B]
    k_step = torch.full((B,), int(k), dtype=torch.int64, device=dev)
    o = select_step(logits, xt_blk, k_step, done, log_prior, sched_t, q_t, cfg_scale=cfg_scale,
                    mask_id=mask_id, stop_id=stop_id, temperature=temperature, top_k=0, top_p=1.0,
                    min_p=0.0, rep_penalty=1.0, history=None, pmi_lambda=1.0, pos_noise=position_noise,
                    use_quantile=use_quantile, gumbel_tok=gumbel_tok, gumbel_pos=gumbel_pos, seed=seed,
                    offset=offset, zero_temp_greedy=True, dense=False, out=out, quantile_lerp=True)
    # a row's block is done once nothing is masked or it holds the stop token
    done_new = done | (o.n_mask_after == 0) | o.hit_eos
    return o.xt, done_new
