"""Parity at the benchmarked sizes: the GPU step against the CPU oracle on the
shapes bench.py runs (configuration 1 at B=64 through a whole 8-step block
evolved by the kernels themselves, configurations 2 and 3 at B=256, and the
engine-buffer mode over consecutive steps), with the kernels' own Philox
noise.  The kernels branch on the number of items per CTA (team sizes, the
on-chip item and request tables), so these shapes run code paths the reduced
cases do not."""
import pytest
import torch

from oracle import select_oracle as O
from tests.parity_util import compare
from yapd_b200.workloads import make_config

pytestmark = pytest.mark.gpu


def _with_philox(inp, seed, offset):
    """The kernels' Philox noise as explicit tensors for the oracle."""
    gt, gp = O.philox_noise(seed, offset, inp.B, inp.L, inp.V)
    inp.gumbel_tok, inp.gumbel_pos = gt, gp
    return inp


def _kw(inp, dev):
    # as bench.py: min-p off everywhere is passed as the scalar (the grouped
    # kernel then runs alone); the reduced tests keep the per-request tensors
    min_p = 0.0 if float(inp.min_p.max()) <= 0.0 else inp.min_p.to(dev)
    return dict(cfg_scale=inp.cfg_scale, mask_id=inp.mask_id, stop_id=inp.stop_id,
                temperature=inp.temperature.to(dev), top_k=inp.top_k.to(dev), top_p=inp.top_p.to(dev),
                min_p=min_p, rep_penalty=inp.rep_penalty.to(dev),
                history=inp.history_bitmap().to(dev), pmi_lambda=inp.pmi_lambda,
                pos_noise=inp.pos_noise, use_quantile=inp.use_quantile)


def _outputs(out):
    return {k: getattr(out, k).cpu() for k in
            ("xt", "sampled", "pmi", "n_unmask", "n_mask_after", "hit_eos", "k_step", "is_commit")}


def _step_and_compare(inp, dev, seed, offset, dense=False):
    from yapd_b200 import select as S
    S.clear_status()
    out = S.select_step(inp.logits.to(dev), inp.xt.to(dev), inp.k_step.to(dev), inp.is_commit.to(dev),
                        inp.log_prior.to(dev), inp.sched_t.to(dev), inp.q_t.to(dev), seed=seed,
                        offset=offset, dense=dense, **_kw(inp, dev))
    torch.cuda.synchronize()
    assert S.read_status() == 0   # no expired wait, no kernel invariant broken
    gpu = _outputs(out)
    _with_philox(inp, seed, offset)
    orc = O.select_step(inp, noise="explicit")
    pos = torch.ones(inp.B, inp.L, dtype=torch.bool) if dense else \
        (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
    n = compare(inp, gpu, orc, inp.gumbel_tok, positions=pos)
    print(f"B={inp.B} L={inp.L} sampled {int(pos.sum())} positions, certified near-ties {n}")
    return gpu, orc


def test_config1_whole_block_b64():
    # configuration 1 as bench.py runs it: 64 requests, all masked at k = 0,
    # eight steps, each step's block state the kernels' own output
    dev = torch.device("cuda")
    inp = make_config(1, seed=101, explicit_noise=False)
    for k in range(inp.num_steps):
        gpu, orc = _step_and_compare(inp, dev, seed=1234, offset=k)
        inp.xt, inp.k_step, inp.is_commit = gpu["xt"], gpu["k_step"], gpu["is_commit"]
    # the block finished: every position unmasked (requests that hit the stop
    # token stay out of the commit phase, server/engine.py:607-609)
    assert not bool((inp.xt == inp.mask_id).any())
    assert bool((inp.is_commit | (inp.xt == inp.stop_id).any(1)).all())


@pytest.mark.parametrize("config", [2, 3])
def test_ragged_b256(config):
    dev = torch.device("cuda")
    inp = make_config(config, seed=202 + config, masked="ragged", explicit_noise=False)
    _step_and_compare(inp, dev, seed=99, offset=config)


def test_config3_engine_buffers_consecutive_steps():
    # continuous batching as bench.py runs it: the kernels gather each block
    # from the token buffer, write it back and advance committing requests
    from yapd_b200 import select as S
    dev = torch.device("cuda")
    inp = make_config(3, seed=303, masked="ragged", explicit_noise=False, commit_frac=0.1)
    B, L = inp.B, inp.L
    nblk = 4
    xt_full = torch.full((B, nblk * L), inp.mask_id, dtype=torch.int64)
    xt_full[:, :L] = inp.xt
    eng = S.EngineBuffers(xt_full=xt_full.to(dev), blk_start=torch.zeros(B, dtype=torch.int64, device=dev),
                          cache_len=torch.zeros(B, dtype=torch.int64, device=dev),
                          n_speech=torch.full((B,), nblk * L, dtype=torch.int64, device=dev),
                          flags=torch.empty(B, 6, dtype=torch.int64, device=dev),
                          blk_limit=(nblk - 1) * L, cache_limit=nblk * L)
    k_d, c_d = inp.k_step.to(dev).clone(), inp.is_commit.to(dev).clone()
    cnt = torch.zeros(1, dtype=torch.int64, device=dev)
    o = S.SelectOutputs.empty(B, L, dev)
    out = S.SelectOutputs(xt=o.xt, sampled=o.sampled, pmi=o.pmi, n_unmask=o.n_unmask,
                          n_mask_after=o.n_mask_after, hit_eos=o.hit_eos, k_step=k_d, is_commit=c_d)
    blk = torch.zeros(B, dtype=torch.int64)
    cache = torch.zeros(B, dtype=torch.int64)
    want_total = 0
    for step in range(3):
        # the oracle's inputs: the block at blk_start of the current buffer
        full = eng.xt_full.cpu()
        inp.xt = full.gather(1, blk[:, None] + torch.arange(L))
        inp.k_step, inp.is_commit = k_d.cpu(), c_d.cpu()
        want_total += int(((inp.xt == inp.mask_id) & ~inp.is_commit[:, None]).sum())
        commit_before = inp.is_commit.clone()
        S.select_step(inp.logits.to(dev), None, k_d, c_d, inp.log_prior.to(dev), inp.sched_t.to(dev),
                      inp.q_t.to(dev), seed=7, offset=step, out=out, engine=eng, L=L,
                      positions_sampled=cnt, **_kw(inp, dev))
        torch.cuda.synchronize()
        _with_philox(inp, 7, step)
        orc = O.select_step(inp, noise="explicit")
        pos = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
        n = compare(inp, _outputs(out), orc, inp.gumbel_tok, positions=pos)
        print(f"step {step}: sampled {int(pos.sum())} positions, certified near-ties {n}")
        xf, blk, cache, fl = O.engine_update(orc, full, blk, cache, eng.n_speech.cpu(), commit_before, L=L,
                                             blk_limit=(nblk - 1) * L, cache_limit=nblk * L)
        if n == 0:
            assert torch.equal(eng.xt_full.cpu(), xf)
            assert torch.equal(eng.flags.cpu(), fl)
        assert torch.equal(eng.blk_start.cpu(), blk)
        assert torch.equal(eng.cache_len.cpu(), cache)
    assert int(cnt.item()) == want_total
