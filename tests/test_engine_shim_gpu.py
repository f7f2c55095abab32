"""The engine shims (FlashEngine._step_gpu select body, TurboEngine._sample) on the GPU
against the CPU oracle with the kernels' Philox noise."""
from types import SimpleNamespace

import pytest
import torch

from oracle import select_oracle as O
from tests.parity_util import compare
from yapd_b200.workloads import make_config

pytestmark = pytest.mark.gpu


def _uniform(inp, T):
    B = inp.B
    inp.temperature = torch.full((B,), T)
    inp.top_k = torch.zeros(B, dtype=torch.int32)
    inp.top_p = torch.ones(B)
    inp.min_p = torch.zeros(B)
    inp.rep_penalty = torch.ones(B)
    inp.history = None
    inp.pmi_lambda = 1.0
    return inp


def test_flash_select_shim():
    from yapd_b200.engine_shim import FlashSelect
    inp = _uniform(make_config(0, seed=5, B=4, L=16, masked="ragged", explicit_noise=False,
                               commit_frac=0.25), 0.6)
    dev = torch.device("cuda")
    B, L = inp.B, inp.L
    e = SimpleNamespace(
        n_branch=2, BS=L, K=inp.num_steps, temp=0.6, tau=0.1, cfg=inp.cfg_scale, posT=5.0,
        MASK=inp.mask_id, STOP=inp.stop_id, V=inp.V, L=L + 64, N_max=L, max_active=B,
        xt=inp.xt.to(dev).clone(), blk_start=torch.zeros(B, dtype=torch.long, device=dev),
        k_step=inp.k_step.to(dev).clone(), cache_len=torch.zeros(B, dtype=torch.long, device=dev),
        n_speech=torch.zeros(B, dtype=torch.long, device=dev), is_commit=inp.is_commit.to(dev).clone(),
        sched_t=inp.sched_t.to(dev), q_t=inp.q_t.to(dev), log_prior=inp.log_prior.to(dev))
    sel = FlashSelect(e, seed=1234)
    blk_idx = e.blk_start[:B, None] + torch.arange(L, device=dev)
    xt_blk = e.xt.gather(1, blk_idx)
    flags, xt_final = sel(inp.logits.to(dev), B, blk_idx, xt_blk, e.is_commit.clone())
    torch.cuda.synchronize()
    orc = O.select_step(inp, noise="philox", seed=1234, offset=0)
    gpu = {"sampled": sel.out.sampled.cpu(), "pmi": sel.out.pmi.cpu(), "xt": xt_final.cpu(),
           "n_mask_after": sel.out.n_mask_after.cpu(), "hit_eos": sel.out.hit_eos.cpu(),
           "k_step": e.k_step.cpu(), "is_commit": e.is_commit.cpu()}
    gt, _ = O.philox_noise(1234, 0, B, L, inp.V)
    pos = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
    compare(inp, gpu, orc, gt, positions=pos)
    assert torch.equal(flags[:, 0].cpu(), inp.is_commit.long())
    assert torch.equal(flags[:, 1].cpu(), orc["n_mask_after"])
    assert torch.equal(e.xt.cpu(), orc["xt_final"])


@pytest.mark.parametrize("gather", [False, True])
def test_engine_writeback(gather):
    # the step writes the engine's token buffer, cache / block offsets and the
    # packed flags (server/engine.py:586-622); with gather=True the kernels also
    # read the block from the token buffer themselves (xt=None)
    from yapd_b200.select import EngineBuffers, SelectOutputs, select_step
    inp = make_config(2, seed=19, B=12, masked="ragged", explicit_noise=False, commit_frac=0.3)
    dev = torch.device("cuda")
    B, L = inp.B, inp.L
    nblk = 5
    g = torch.Generator().manual_seed(3)
    blk = torch.randint(0, nblk, (B,), generator=g)
    blk[0] = nblk - 1                       # a row at the last block: blk_start clamps
    blk_start = blk * L
    xt_full = torch.randint(0, 6561, (B, nblk * L), generator=g)
    xt_full.scatter_(1, blk_start[:, None] + torch.arange(L), inp.xt)
    cache_len = blk_start + 7
    cache_len[1] = 10 * L                   # at the cache limit: clamps
    n_speech = torch.randint(0, 500, (B,), generator=g)
    eng = EngineBuffers(xt_full=xt_full.to(dev), blk_start=blk_start.to(dev), cache_len=cache_len.to(dev),
                        n_speech=n_speech.to(dev), flags=torch.empty(B, 6, dtype=torch.int64, device=dev),
                        blk_limit=(nblk - 1) * L, cache_limit=10 * L)
    out = SelectOutputs.empty(B, L, dev)
    select_step(inp.logits.to(dev), None if gather else inp.xt.to(dev), inp.k_step.to(dev),
                inp.is_commit.to(dev), inp.log_prior.to(dev), inp.sched_t.to(dev), inp.q_t.to(dev),
                cfg_scale=inp.cfg_scale, mask_id=inp.mask_id, stop_id=inp.stop_id,
                temperature=inp.temperature.to(dev), top_k=inp.top_k.to(dev), top_p=inp.top_p.to(dev),
                min_p=inp.min_p.to(dev), rep_penalty=inp.rep_penalty.to(dev),
                history=inp.history_bitmap().to(dev), pmi_lambda=inp.pmi_lambda, seed=5, offset=1,
                out=out, engine=eng, L=L)
    torch.cuda.synchronize()
    orc = O.select_step(inp, noise="philox", seed=5, offset=1)
    gt, _ = O.philox_noise(5, 1, B, L, inp.V)
    gpu = {k: getattr(out, k).cpu() for k in ("xt", "sampled", "pmi", "n_mask_after", "hit_eos", "k_step",
                                              "is_commit")}
    pos = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
    assert compare(inp, gpu, orc, gt, positions=pos) == 0
    xf, bs, cl, fl = O.engine_update(orc, xt_full, blk_start, cache_len, n_speech, inp.is_commit, L=L,
                                     blk_limit=(nblk - 1) * L, cache_limit=10 * L)
    assert torch.equal(eng.xt_full.cpu(), xf)
    assert torch.equal(eng.blk_start.cpu(), bs)
    assert torch.equal(eng.cache_len.cpu(), cl)
    assert torch.equal(eng.flags.cpu(), fl)


def test_turbo_sample_shim():
    from yapd_b200.engine_shim import turbo_sample
    from oracle import philox
    g = torch.Generator().manual_seed(11)
    R, V = 48, 6563
    logits = torch.randn(R, V, generator=g) * 2
    seen = torch.rand(R, V, generator=g) < 0.03
    e = SimpleNamespace(temp=0.8, top_k=1000, top_p=0.95, rep_p=1.2, _yapd_seed=77)
    got = turbo_sample(e, logits.cuda(), seen.cuda()).cpu()
    G = O.gumbel_from_uniform(philox.token_uniforms(77, 0, R, 1, V)).view(R, V)
    one = torch.ones(R)
    want = O.sample_tokens(logits, 0.8 * one, torch.full((R,), 1000, dtype=torch.int32),
                           0.95 * one, torch.zeros(R), 1.2 * one, seen, G, zero_temp="unscaled")
    assert torch.equal(got, want)
