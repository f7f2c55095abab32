"""Generate the select-step golden fixtures from the unmodified reference.

Run where an m8than/yapd source checkout is available (its location in
``$YAPD_REFERENCE_ROOT``, else ``ref_loader.REF_ROOT``'s default):

    python -m tests.golden.make_golden

For every case of ``tests/golden/cases.py`` it drives the reference's own
code (``ref_loader.py``) and writes ``tests/golden/<case>.npz`` holding:

* ``sampled``  (B, L) int32 — the token the reference samples at each position;
* ``pmi_ranked`` (B, L) f32 — the reference's ``where(is_mask, pmi, -inf)``,
  i.e. the noisy PMI it ranks masked positions by (``server/engine.py:581``);
* ``xt_final`` (B, L) int64, ``flags`` (B, 6) int64, ``k_step`` (B,) int64 —
  the reference's step outputs (``server/engine.py:586-622``);
* ``digest`` — SHA-256 of the regenerated inputs.

Unfiltered cases run ``FlashEngine._step_gpu`` directly.  Filter-chain cases
draw each request's samples with ``TurboEngine._sample`` on the CFG-guided
rows and then push those samples through ``_step_gpu`` with forcing noise, so
PMI, ranking and unmask also come from the reference.  The ``lambda_half``
case takes its PMI from ``calibration.compute_pmi`` and
``cfg_guidance.pmi_cfg_combine`` (the engine hard-codes lambda = 1).
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases, ref_loader as R  # noqa: E402


def filtered_rows(inp) -> bool:
    return bool(((inp.top_k > 0) & (inp.top_k < inp.V)).any() or (inp.top_p < 1).any()
                or (inp.min_p > 0).any()
                or (inp.history is not None and (inp.rep_penalty != 1).any()))


def reference_samples(inp) -> torch.Tensor:
    """Per-request ``TurboEngine._sample`` over the CFG-guided rows."""
    B, L, V = inp.B, inp.L, inp.V
    if inp.nb == 2:
        guided = R.reference_guided(inp)
    else:
        guided = inp.logits.float()
    out = torch.empty(B, L, dtype=torch.long)
    for b in range(B):
        seen = (inp.history[b].expand(L, V).clone() if inp.history is not None
                else torch.zeros(L, V, dtype=torch.bool))
        out[b] = R.run_turbo_sample(guided[b], seen, inp.gumbel_tok[b],
                                    float(inp.temperature[b]), int(inp.top_k[b]),
                                    float(inp.top_p[b]), float(inp.rep_penalty[b]))
    return out


def run_case(name: str) -> dict:
    inp = cases.build(name)
    tau = inp.meta.get("tau", 0.1)
    pos_temp = 5.0 if inp.pos_noise else 0.0
    if filtered_rows(inp) or name == "lambda_half":
        sampled = reference_samples(inp)
        g_tok = R.forcing_noise(sampled, inp.V)
        temp = 1.0
    else:
        sampled = None
        g_tok = inp.gumbel_tok
        temps = inp.temperature.unique()
        assert temps.numel() == 1
        temp = float(temps[0])
    with R.record_internals() as rec:
        flags, xt_final, k_step = R.run_flash_step(inp, g_tok, inp.gumbel_pos, temp,
                                                   pos_temp=pos_temp, tau=tau)
    if sampled is None:
        sampled = rec.argmax[0]
    else:
        assert torch.equal(rec.argmax[0], sampled)
    out = dict(sampled=sampled.numpy().astype(np.int32),
               pmi_ranked=rec.argsort_in[0].numpy().astype(np.float32),
               xt_final=xt_final.numpy(), flags=flags.numpy(), k_step=k_step.numpy())
    if name == "lambda_half":
        R.load()
        from chatterbox_flash.calibration import compute_pmi
        from chatterbox_flash.cfg_guidance import pmi_cfg_combine
        B, L, V = inp.B, inp.L, inp.V
        lc = inp.logits.float().view(B, 2, L, V)
        prior = inp.meta["prior"]
        pmis = []
        for b in range(B):
            pc = torch.softmax(lc[b, 0], -1)
            pu = torch.softmax(lc[b, 1], -1)
            p_c = compute_pmi(pc, sampled[b], marginal_prior=prior, prior_lambda=inp.pmi_lambda)
            p_u = compute_pmi(pu, sampled[b], marginal_prior=prior, prior_lambda=inp.pmi_lambda)
            pmis.append(pmi_cfg_combine(p_c, p_u, inp.cfg_scale))
        pmi = torch.stack(pmis)
        is_mask = inp.xt == inp.mask_id
        pmi = torch.where(is_mask, pmi + inp.gumbel_pos, pmi)
        out["pmi_lambda"] = pmi.numpy().astype(np.float32)
        # the engine's unmask/PMI ran with lambda = 1: keep only sampled + pmi_lambda
        for k in ("pmi_ranked", "xt_final", "flags", "k_step"):
            out.pop(k)
    out["digest"] = np.array(cases.input_digest(inp))
    out["torch_version"] = np.array(torch.__version__)
    return out


def main():
    if not R.reference_available():
        raise SystemExit(f"reference checkout not found at {R.REF_ROOT}")
    summary = {}
    for name in cases.REFERENCE_CASES:
        out = run_case(name)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        summary[name] = {k: list(v.shape) for k, v in out.items() if v.ndim}
        print(name, "ok")
    with open(os.path.join(HERE, "MANIFEST.json"), "w") as f:
        json.dump({"cases": summary, "torch": torch.__version__}, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
