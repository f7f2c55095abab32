"""Fixtures of the offline generator's block step from the unmodified reference.

    python -m tests.golden.make_offline_golden

For every case of ``offline_cases.py`` it calls the reference's own
``_pmi_count_early_step_unmask`` (``chatterbox_flash/model.py:185-311``) row by
row, as ``ChatterboxFlashT3.generate`` does (``model.py:862-906``), with
``temperature_sampling="gumbel"`` and the global RNG seeded so that its draws
are the case's noise, and writes ``tests/golden/<case>.npz``: ``xt`` (B, bl)
after the step and ``done`` (B,) (``n_mask == 0`` or the stop token).
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import offline_cases as OC, ref_loader as R  # noqa: E402


def run_case(name: str) -> dict:
    c = OC.build(name)
    R.load()
    import chatterbox_flash.model as M
    from chatterbox_flash.cfg_guidance import apply_zero_text_cfg_from_logits
    B, bl, K, k = c["B"], c["bl"], c["K"], c["k"]
    w = c["cfg_scale"]
    lc = c["logits_c"].float()
    if w != 0.0:
        lu = c["logits_u"].float()
        blk_logits = apply_zero_text_cfg_from_logits(lc, lu, w)
        pc, pu = torch.softmax(lc, -1), torch.softmax(lu, -1)
    else:
        blk_logits, pc, pu = lc, None, None
    xt = c["xt"].clone()
    done = c["done"].clone()
    torch.manual_seed(c["noise_seed"])
    for b in range(B):
        if bool(done[b]):
            continue
        r = M._pmi_count_early_step_unmask(
            blk_logits[b], xt[b], bl=bl, k=k, K=K, MASK=OC.MASK, device=torch.device("cpu"),
            temperature=c["temperature"], temperature_sampling="gumbel",
            omnivoice_unmask_schedule_k=c["sched"][k], time_shift_tau=c["time_shift_tau"],
            prior_override_v=c["prior"], block_marginal_prior=None,
            pmi_cfg_probs_c_bl=None if pc is None else pc[b], pmi_cfg_probs_u_bl=None if pu is None else pu[b],
            cfg_scale_for_pmi=w, position_temperature=c["position_temperature"])
        xt[b] = r["xt_step"]
        if r["n_mask"] == 0 or bool((xt[b] == OC.STOP).any()):
            done[b] = True
    return dict(xt=xt.numpy(), done=done.numpy(), torch_version=np.array(torch.__version__))


def main():
    if not R.reference_available():
        raise SystemExit(f"reference checkout not found at {R.REF_ROOT}")
    for name in OC.CASES:
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **run_case(name))
        print(name, "ok")


if __name__ == "__main__":
    main()
