"""Failure detection on the device without a fault: bounded pipeline waits
that run out.

With ``wait_limit_ns < 0`` every pipeline wait gives up at once (the final
drain of in-flight copies still waits with the default limit, so no copy
outlives its CTA).  The kernels must return, record
``YAPD_STATUS_WAIT_TIMEOUT``, leave every position they had to sample at -2
with its request's state unchanged (``YAPD_STATUS_ROWS_SKIPPED``), and the
next call with the default limit must be exact again."""
import pytest
import torch

from oracle import select_oracle as O
from tests.parity_util import compare, run_gpu
from yapd_b200 import _native as N
from yapd_b200 import select as S
from yapd_b200.workloads import make_config

pytestmark = pytest.mark.gpu


def _run(inp, dev, min_p=None, **kw):
    out = S.select_step(
        inp.logits.to(dev), inp.xt.to(dev), inp.k_step.to(dev), inp.is_commit.to(dev), inp.log_prior.to(dev),
        inp.sched_t.to(dev), inp.q_t.to(dev), cfg_scale=inp.cfg_scale, mask_id=inp.mask_id,
        stop_id=inp.stop_id, temperature=inp.temperature.to(dev), top_k=inp.top_k.to(dev),
        top_p=inp.top_p.to(dev), min_p=inp.min_p.to(dev) if min_p is None else min_p, rep_penalty=inp.rep_penalty.to(dev),
        history=inp.history_bitmap().to(dev), pmi_lambda=inp.pmi_lambda, gumbel_tok=inp.gumbel_tok.to(dev),
        gumbel_pos=inp.gumbel_pos.to(dev), **kw)
    torch.cuda.synchronize()
    return {k: getattr(out, k).cpu() for k in
            ("xt", "sampled", "pmi", "n_unmask", "n_mask_after", "hit_eos", "k_step", "is_commit")}


# configuration 1: the bf16 warp kernel; 3: its grouped pipeline (histogram
# select); 3 with the scalar min-p 0: the bf16 grouped kernel launched alone;
# 2: the fp32 sample kernel
@pytest.mark.parametrize("config,scalar_minp", [(1, False), (3, False), (3, True), (2, False)])
def test_expired_wait_is_reported_and_contained(config, scalar_minp):
    dev = torch.device("cuda")
    inp = make_config(config, seed=11, B=16, masked="ragged", commit_frac=0.2)
    if scalar_minp:
        assert float(inp.min_p.max()) <= 0.0
    S.clear_status()
    got = _run(inp, dev, min_p=0.0 if scalar_minp else None, wait_limit_ns=-1)
    st = S.read_status()
    assert st & N.YAPD_STATUS_WAIT_TIMEOUT
    orc = O.select_step(inp, noise="explicit")
    want = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
    smp = got["sampled"]
    assert bool((smp[want] == -2).all())
    assert bool((smp[~want] == -1).all())
    assert st & N.YAPD_STATUS_ROWS_SKIPPED
    # every request keeps its state: a denoising request with masked positions
    # is skipped, and the others have nothing that depends on the samples
    rows = want.any(1)
    for b in range(inp.B):
        if bool(rows[b]):
            assert torch.equal(got["xt"][b], inp.xt[b])
            assert int(got["k_step"][b]) == int(inp.k_step[b])
            assert int(got["n_unmask"][b]) == 0
            assert not bool(got["is_commit"][b])
    # the next call with the default limit is exact and reports nothing
    S.clear_status()
    gpu = run_gpu(inp, dense=False)
    assert S.read_status() == 0
    assert compare(inp, gpu, orc, inp.gumbel_tok, positions=want) == 0


def test_expired_wait_sample_rows():
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(5)
    R, V = 64, 6563
    logits = torch.randn(R, V, generator=g) * 2
    G = O.gumbel_from_uniform(torch.rand(R, V, generator=g))
    one = torch.ones(R)
    kw = dict(temperature=(0.8 * one).to(dev), top_k=torch.full((R,), 1000, dtype=torch.int32, device=dev),
              top_p=(0.95 * one).to(dev), min_p=torch.zeros(R, device=dev), rep_penalty=one.to(dev),
              gumbel=G.to(dev))
    S.clear_status()
    S.sample_rows(logits.to(dev), wait_limit_ns=-1, **kw)
    torch.cuda.synchronize()
    assert S.read_status() & N.YAPD_STATUS_WAIT_TIMEOUT
    S.clear_status()
    got = S.sample_rows(logits.to(dev), **kw).cpu().long()
    assert S.read_status() == 0
    want = O.sample_tokens(logits, 0.8 * one, torch.full((R,), 1000, dtype=torch.int32), 0.95 * one,
                           torch.zeros(R), one, None, G, zero_temp="unscaled")
    assert torch.equal(got, want)
