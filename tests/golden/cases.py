"""Seeded select-step cases shared by the fixture generator and the tests.

Each case regenerates its inputs deterministically from a seed (CPU
``torch.Generator``), so fixtures only store outputs plus an input checksum.
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from yapd_b200.workloads import (StepInputs, make_config, omnivoice_unmask_schedule,
                                 quantile_table)


def _set_uniform(inp: StepInputs, *, T=0.8, top_k=0, top_p=1.0, min_p=0.0, rep=1.0):
    B = inp.B
    inp.temperature = torch.full((B,), float(T))
    inp.top_k = torch.full((B,), int(top_k), dtype=torch.int32)
    inp.top_p = torch.full((B,), float(top_p))
    inp.min_p = torch.full((B,), float(min_p))
    inp.rep_penalty = torch.full((B,), float(rep))
    return inp


def _prior_from_probs(inp: StepInputs, seed: int):
    """``log_prior = log(clamp(prior, 1e-8))`` as ``server/engine.py:363-366``
    builds it, so calibration's lambda-PMI is reproducible from ``prior``."""
    g = torch.Generator().manual_seed(seed + 77)
    prior = torch.softmax(torch.randn(inp.V, generator=g), -1).clamp_min(1e-8)
    inp.log_prior = prior.log()
    inp.meta["prior"] = prior
    return inp


def _steps(inp: StepInputs, K: int, tau: float = 0.1, t_shift: float = 0.5):
    inp.num_steps = K
    inp.sched_t = torch.tensor(omnivoice_unmask_schedule(inp.L, K, t_shift), dtype=torch.long)
    inp.q_t = torch.tensor(quantile_table(K, tau), dtype=torch.float32)
    inp.use_quantile = tau > 0
    inp.meta["tau"] = tau
    return inp


def build(name: str) -> StepInputs:
    """Named case -> inputs (explicit noise included)."""
    if name == "flash_c0":
        inp = make_config(0, seed=11)
        _set_uniform(inp, T=0.8)
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "flash_ragged":
        inp = make_config(2, seed=12, B=8, L=16, masked="ragged", commit_frac=0.25)
        _steps(inp, 10)
        inp.k_step = inp.k_step.clamp(max=9)
        _set_uniform(inp, T=0.6)
        inp.cfg_scale = 1.0
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "flash_nocfg":
        full = make_config(0, seed=13, B=4, L=16)
        full.logits = full.logits.view(4, 2, 16, -1)[:, 0].contiguous()
        full.nb = 1
        full.cfg_scale = 0.0
        inp = _set_uniform(full, T=0.7)
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "flash_bf16":
        inp = make_config(1, seed=14, B=2, L=16, masked="ragged")
        _set_uniform(inp, T=0.8)
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "flash_tau0_last":
        inp = make_config(0, seed=15, B=4, L=16, masked="ragged")
        _steps(inp, 4, tau=0.0)
        inp.k_step = torch.tensor([0, 1, 2, 3])
        _set_uniform(inp, T=1.0)
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "flash_edge_masks":
        inp = make_config(0, seed=16, B=4, L=16)
        inp.xt[0] = torch.arange(16) + 100          # nothing masked
        inp.xt[1, 1:] = torch.arange(15) + 200      # one masked
        inp.xt[2, :8] = 6562                        # STOP present
        _set_uniform(inp, T=0.8)
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "chain_c0":
        inp = make_config(0, seed=21, B=2, L=16)
        _set_uniform(inp, T=0.8, top_p=0.95, rep=1.2)
        inp.pmi_lambda = 1.0
    elif name == "chain_topk":
        inp = make_config(0, seed=22, B=4, L=8)
        _set_uniform(inp, T=1.1, top_k=50, top_p=0.9, rep=1.3)
        inp.pmi_lambda = 1.0
    elif name == "chain_topk_only":
        inp = make_config(0, seed=23, B=4, L=8)
        _set_uniform(inp, T=0.9, top_k=200)
        inp.pmi_lambda = 1.0
        inp.history = None
    elif name == "chain_per_request":
        inp = make_config(2, seed=24, B=8, L=8, masked="ragged")
        inp.pmi_lambda = 1.0
    elif name == "chain_bf16":
        inp = make_config(3, seed=25, B=4, L=8, masked="ragged")
        inp.pmi_lambda = 1.0
    elif name == "lambda_half":
        inp = make_config(0, seed=26, B=2, L=16)
        _set_uniform(inp, T=0.8, top_p=0.95, rep=1.2)
        _prior_from_probs(inp, 26)
        inp.pmi_lambda = 0.5
    else:
        raise KeyError(name)
    inp.meta["case"] = name
    return inp


REFERENCE_CASES = [
    "flash_c0", "flash_ragged", "flash_nocfg", "flash_bf16", "flash_tau0_last",
    "flash_edge_masks", "chain_c0", "chain_topk", "chain_topk_only", "chain_per_request",
    "chain_bf16", "lambda_half",
]


def input_digest(inp: StepInputs) -> str:
    """SHA-256 over the input tensors, to catch generator drift."""
    h = hashlib.sha256()
    for t in (inp.logits, inp.xt, inp.k_step, inp.is_commit, inp.log_prior, inp.temperature,
              inp.top_k, inp.top_p, inp.rep_penalty, inp.gumbel_tok, inp.gumbel_pos,
              inp.history):
        if t is None:
            h.update(b"none")
            continue
        a = t.detach().cpu()
        if a.dtype == torch.bfloat16:
            a = a.view(torch.int16)
        h.update(np.ascontiguousarray(a.numpy()).tobytes())
    return h.hexdigest()
