"""Seeded cases of the offline generator's block step (shared by the fixture
generator and the tests).  Each case regenerates its inputs from a seed and
the reference's noise from a second seed, drawn in the order
``_pmi_count_early_step_unmask`` draws it (``chatterbox_flash/model.py:76-80``:
per row, the token uniforms ``(bl, V)`` when ``temperature > 0``, then the
position uniforms ``(bl,)`` when ``position_temperature > 0``)."""
from __future__ import annotations

import torch

from oracle.select_oracle import offline_gumbel
from yapd_b200.workloads import make_logits, omnivoice_unmask_schedule, quantile_table

V = 8194
MASK = V
STOP = 6562

# name: (B, bl, K, k, cfg_scale, temperature, position_temperature, time_shift_tau, done rows)
CASES = {
    "offline_cfg": (6, 16, 10, 2, 1.0, 0.6, 5.0, 0.1, ()),
    "offline_nocfg_last": (5, 16, 10, 9, 0.0, 0.6, 5.0, 0.1, ()),
    "offline_greedy": (4, 32, 8, 0, 1.0, 0.0, 5.0, 0.1, (2,)),
    "offline_tau0": (6, 16, 10, 4, 1.0, 0.8, 0.0, 0.0, ()),
}


def build(name: str):
    B, bl, K, k, w, T, posT, tau, done_rows = CASES[name]
    seed = sum(map(ord, name))
    g = torch.Generator().manual_seed(seed)
    logits_c = make_logits(g, B, bl, V)
    logits_u = make_logits(g, B, bl, V) if w != 0.0 else None
    prior = torch.softmax(torch.randn(V, generator=g), -1)
    xt = torch.randint(0, 6561, (B, bl), generator=g)
    for b in range(B):
        n = int(torch.randint(1, bl + 1, (1,), generator=g))
        xt[b, torch.randperm(bl, generator=g)[:n]] = MASK
    done = torch.zeros(B, dtype=torch.bool)
    for b in done_rows:
        done[b] = True
    # the reference's uniforms, in its draw order (rows not done only)
    gn = torch.Generator().manual_seed(seed + 1)
    G = torch.zeros(B, bl, V)
    Gpos = torch.zeros(B, bl)
    for b in range(B):
        if bool(done[b]):
            continue
        if T > 0:
            G[b] = offline_gumbel(torch.rand(bl, V, generator=gn))
        if posT > 0:
            Gpos[b] = offline_gumbel(torch.rand(bl, generator=gn))
    sched = omnivoice_unmask_schedule(bl, K, 0.5)
    q = quantile_table(K, tau) if tau > 0 else [0.0] * K
    return dict(name=name, B=B, bl=bl, K=K, k=k, cfg_scale=w, temperature=T, position_temperature=posT,
                time_shift_tau=tau, logits_c=logits_c, logits_u=logits_u, prior=prior, xt=xt, done=done,
                G=G, Gpos=Gpos, sched=sched, q=q, noise_seed=seed + 1)
