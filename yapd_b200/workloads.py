"""Seeded synthetic inputs for the block-diffusion select step.

The reference publishes no dataset for this path; its inputs are the speech-head
logits of a live model.  These generators stand in for them with the value
distributions the benchmark configurations name:

* logits ~ N(0, 2) (std 2) with three tokens per row boosted by +8,
* log-prior = log_softmax(N(0, 1)) over the vocabulary,
* a uniform-random repetition history per request,
* block state (``xt``, ``k_step``, ``is_commit``) of a running block.

Everything is generated with ``torch.Generator`` seeded on the CPU, so a test
on one machine and the CPU oracle on another see bit-identical tensors.

Constants follow the reference engine: the vocabulary size ``V = 8194`` and
``MASK = V`` (``server/engine.py:313``, ``:317``), ``STOP = 6562``
(``server/engine_ar.py:154``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

V_SPEECH = 8194
MASK_ID = V_SPEECH
STOP_ID = 6562


def omnivoice_unmask_schedule(n_total_mask: int, num_steps: int, t_shift: float) -> list[int]:
    """Per-step unmask counts of the time-shifted ``r_n`` curve.

    Follows ``chatterbox_flash/model.py:133-177``: cumulative fraction
    ``r(s) = t*s / (1 + (t-1)*s)`` at ``s = step/K``, converted to integer
    counts by cumulative rounding, the last step taking the remainder.
    """
    K = max(1, int(num_steps))
    N = max(0, int(n_total_mask))
    if N == 0:
        return [0] * K
    if K == 1:
        return [N]
    tau = float(t_shift)
    if tau <= 0:
        base = N // K
        out = [base] * K
        out[-1] += N - sum(out)
        return out
    fracs = [tau * (s / K) / (1.0 + (tau - 1.0) * (s / K)) for s in range(K + 1)]
    counts: list[int] = []
    done = 0
    left = N
    for s in range(K):
        if s == K - 1:
            num = left
        else:
            num = min(max(0, int(round(N * fracs[s + 1])) - done), left)
        counts.append(num)
        done += num
        left -= num
    return counts


def quantile_table(num_steps: int, time_shift_tau: float) -> list[float]:
    """``q_k = max(0, 1 - tau*(k+1)/K)`` as built in ``server/engine.py:357``."""
    K = int(num_steps)
    return [max(0.0, 1.0 - time_shift_tau * (k + 1) / K) for k in range(K)]


def history_to_bitmap(history: torch.Tensor) -> torch.Tensor:
    """Pack a ``(B, V)`` bool history into ``(B, ceil(V/32))`` int32 words.

    Bit ``v & 31`` of word ``v >> 5`` is set when token ``v`` is in the history.
    """
    B, V = history.shape
    W = (V + 31) // 32
    pad = torch.zeros(B, W * 32, dtype=torch.int64, device=history.device)
    pad[:, :V] = history.to(torch.int64)
    shifts = torch.arange(32, dtype=torch.int64, device=history.device)
    words = (pad.view(B, W, 32) << shifts).sum(-1)
    words = torch.where(words >= 2**31, words - 2**32, words)
    return words.to(torch.int32)


@dataclass
class StepInputs:
    """One select step's inputs in the layout the engine holds them.

    ``logits`` is ``(B*nb, L, V)`` with rows ``b*nb`` (conditional) and
    ``b*nb + 1`` (unconditional), as ``FlashEngine._build_prefixes``
    interleaves them (``server/engine.py:397-401``).
    """
    logits: torch.Tensor
    xt: torch.Tensor
    k_step: torch.Tensor
    is_commit: torch.Tensor
    log_prior: torch.Tensor
    sched_t: torch.Tensor
    q_t: torch.Tensor
    temperature: torch.Tensor
    top_k: torch.Tensor
    top_p: torch.Tensor
    min_p: torch.Tensor
    rep_penalty: torch.Tensor
    history: torch.Tensor | None
    cfg_scale: float
    pmi_lambda: float
    pos_noise: bool
    use_quantile: bool
    num_steps: int
    nb: int
    mask_id: int = MASK_ID
    stop_id: int = STOP_ID
    gumbel_tok: torch.Tensor | None = None
    gumbel_pos: torch.Tensor | None = None
    meta: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return self.xt.shape[0]

    @property
    def L(self) -> int:
        return self.xt.shape[1]

    @property
    def V(self) -> int:
        return self.logits.shape[-1]

    def history_bitmap(self) -> torch.Tensor | None:
        return None if self.history is None else history_to_bitmap(self.history)


def make_logits(gen: torch.Generator, rows: int, L: int, V: int, std: float = 2.0,
                boost: float = 8.0, n_boost: int = 3, dtype=torch.float32) -> torch.Tensor:
    """``(rows, L, V)`` logits ~ N(0, std) with ``n_boost`` tokens per row +``boost``."""
    x = torch.randn(rows, L, V, generator=gen) * std
    if n_boost > 0:
        idx = torch.randint(0, V, (rows, L, n_boost), generator=gen)
        x.scatter_add_(2, idx, torch.full(idx.shape, boost))
    return x.to(dtype)


def make_log_prior(gen: torch.Generator, V: int) -> torch.Tensor:
    return torch.log_softmax(torch.randn(V, generator=gen), dim=-1)


def make_history(gen: torch.Generator, B: int, V: int, lengths) -> torch.Tensor:
    """Bool ``(B, V)`` history; request b holds ``lengths[b]`` uniform draws."""
    hist = torch.zeros(B, V, dtype=torch.bool)
    for b in range(B):
        n = int(lengths[b])
        if n > 0:
            hist[b, torch.randint(0, V, (n,), generator=gen)] = True
    return hist


def make_block_state(gen: torch.Generator, B: int, L: int, K: int, mask_id: int, V: int,
                     masked_counts=None, k_steps=None, commit_frac: float = 0.0):
    """Block tokens with ``masked_counts[b]`` random positions still ``MASK``."""
    if masked_counts is None:
        masked_counts = [L] * B
    xt = torch.randint(0, min(V, 6561), (B, L), generator=gen)
    for b in range(B):
        m = int(masked_counts[b])
        pos = torch.randperm(L, generator=gen)[:m]
        xt[b, pos] = mask_id
    if k_steps is None:
        k_step = torch.zeros(B, dtype=torch.long)
    else:
        k_step = torch.as_tensor(k_steps, dtype=torch.long).clone()
    is_commit = torch.rand(B, generator=gen) < commit_frac
    return xt, k_step, is_commit


def make_config(config: int, seed: int = 0, *, B: int | None = None, L: int | None = None,
                V: int = V_SPEECH, dtype=None, explicit_noise: bool = True,
                masked: str = "all", k_step: int | None = None,
                commit_frac: float = 0.0, lmhead_logits: bool = True) -> StepInputs:
    """Inputs for benchmark configurations 0-3.

    * 0: B=1, L=16, fp32, uniform parameters (the CPU parity case).
    * 1: B=64, L=32, bf16, uniform parameters.
    * 2: B=256, L=32, fp32, ragged masks and per-request parameters.
    * 3: B=256 per GPU, L=32, bf16, config-2 parameters.
    * 4: B=512, L=32, bf16 logits of a speech LM head: hidden states
      ``(B*2*L, 1024)`` ~ N(0, 1) times a head weight ``(V, 1024)`` ~ N(0, 0.02)
      (both bf16, fp32 accumulation, rounded to bf16), config-1 parameters.
      ``meta["hidden"]`` and ``meta["weight"]`` hold the two operands;
      ``lmhead_logits=False`` skips the host GEMM (``logits`` is then a
      zero-stride view of the right shape, for callers that run the GEMM on
      the device).

    ``masked``: "all" (a block's first step) or "ragged" (U{1..L} masked
    positions per request).  ``B``, ``L``, ``V`` and ``dtype`` override the
    configuration's sizes for smaller parity cases.
    """
    gen = torch.Generator().manual_seed(int(seed) * 1000003 + config)
    defaults = {0: (1, 16, torch.float32, 4), 1: (64, 32, torch.bfloat16, 8),
                2: (256, 32, torch.float32, 8), 3: (256, 32, torch.bfloat16, 8),
                4: (512, 32, torch.bfloat16, 8)}
    B0, L0, dt0, K = defaults[config]
    B = B0 if B is None else B
    L = L0 if L is None else L
    dtype = dt0 if dtype is None else dtype
    nb = 2
    cfg_scale = 0.5
    pmi_lambda = 0.5
    meta = {"config": config, "seed": seed}
    if config == 4:
        hidden, weight = make_lmhead(gen, B * nb * L, V)
        meta.update(hidden=hidden, weight=weight)
        if lmhead_logits:
            logits = lmhead_logits_of(hidden, weight).view(B * nb, L, V).to(dtype)
        else:
            logits = torch.zeros((1, 1, 1), dtype=dtype).expand(B * nb, L, V)
    else:
        logits = make_logits(gen, B * nb, L, V, dtype=dtype)
    log_prior = make_log_prior(gen, V)
    if config in (0, 1, 4):
        temperature = torch.full((B,), 0.8)
        top_k = torch.zeros(B, dtype=torch.int32)
        top_p = torch.full((B,), 0.95)
        min_p = torch.full((B,), 0.05)
        rep = torch.full((B,), 1.2)
        hist_len = [256] * B
    else:
        temperature = 0.5 + 0.7 * torch.rand(B, generator=gen)
        choices = torch.tensor([0, 50, 200, 1000], dtype=torch.int32)
        top_k = choices[torch.randint(0, 4, (B,), generator=gen)]
        top_p = 0.8 + 0.2 * torch.rand(B, generator=gen)
        min_p = torch.zeros(B)
        rep = 1.0 + 0.5 * torch.rand(B, generator=gen)
        hist_len = torch.randint(0, 2049, (B,), generator=gen).tolist()
    history = make_history(gen, B, V, hist_len)
    if masked == "all":
        counts = [L] * B
    else:
        counts = torch.randint(1, L + 1, (B,), generator=gen).tolist()
    ks = None if k_step is None else [k_step] * B
    if masked == "ragged" and k_step is None:
        ks = torch.randint(0, K, (B,), generator=gen).tolist()
    xt, k_steps, is_commit = make_block_state(gen, B, L, K, MASK_ID if V == V_SPEECH else V, V,
                                              masked_counts=counts, k_steps=ks,
                                              commit_frac=commit_frac)
    sched = omnivoice_unmask_schedule(L, K, 0.5)
    q = quantile_table(K, 0.1)
    gtok = gpos = None
    if explicit_noise:
        gtok = gumbel_from_uniform(torch.rand(B, L, V, generator=gen))
        gpos = gumbel_from_uniform(torch.rand(B, L, generator=gen))
    return StepInputs(
        logits=logits, xt=xt, k_step=k_steps, is_commit=is_commit, log_prior=log_prior,
        sched_t=torch.tensor(sched, dtype=torch.long), q_t=torch.tensor(q, dtype=torch.float32),
        temperature=temperature.float(), top_k=top_k, top_p=top_p.float(), min_p=min_p.float(),
        rep_penalty=rep.float(), history=history, cfg_scale=cfg_scale, pmi_lambda=pmi_lambda,
        pos_noise=True, use_quantile=True, num_steps=K, nb=nb,
        mask_id=MASK_ID if V == V_SPEECH else V, stop_id=STOP_ID if V > STOP_ID else V - 1,
        gumbel_tok=gtok, gumbel_pos=gpos, meta=meta)


LMHEAD_HIDDEN = 1024


def make_lmhead(gen: torch.Generator, rows: int, V: int, H: int = LMHEAD_HIDDEN):
    """Speech-head operands: hidden ``(rows, H)`` ~ N(0, 1) and weight
    ``(V, H)`` ~ N(0, 0.02), both bf16 (the config-4 distributions)."""
    hidden = torch.randn(rows, H, generator=gen).to(torch.bfloat16)
    weight = (torch.randn(V, H, generator=gen) * 0.02).to(torch.bfloat16)
    return hidden, weight


def lmhead_logits_of(hidden: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """``hidden @ weight.T`` accumulated in fp32, rounded to bf16 (the
    speech head of ``server/engine.py:517-520``)."""
    return (hidden.float() @ weight.float().T).to(torch.bfloat16)


def gumbel_from_uniform(u: torch.Tensor) -> torch.Tensor:
    """Standard Gumbel noise from uniforms, with the clamps of
    ``server/engine.py:88-91``: ``-log(max(-log(max(u,1e-20)),1e-20))``."""
    u = u.clamp_min(1e-20)
    return -torch.log((-torch.log(u)).clamp_min(1e-20))


def algorithmic_bytes(inp: StepInputs, rows_sampled: int, positions_sampled: int,
                      explicit_noise: bool) -> int:
    """Bytes the select step must move for one step (the roofline numerator).

    logits rows read + log-prior + history bitmaps (when a penalty is on) +
    per-position state (xt in/out 16 B, sampled id and PMI 8 B) + per-request
    parameters; plus the explicit Gumbel rows in explicit-noise mode.
    """
    s = inp.logits.element_size()
    V = inp.V
    b = rows_sampled * V * s + 4 * V
    if inp.history is not None and bool((inp.rep_penalty != 1.0).any()):
        b += inp.B * math.ceil(V / 32) * 4
    b += inp.B * inp.L * (16 + 8) + inp.B * 32
    if explicit_noise:
        b += positions_sampled * (4 * V + 4)
    return b
