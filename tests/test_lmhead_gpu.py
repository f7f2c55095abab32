"""Fused speech head + select step (``yapd_lmhead_select_step``) on the GPU.

Parity is in two parts.  (1) The tensor-core GEMM: the fp32 logits the
epilogue consumed (written out through ``logits_out``) against an fp64
``hidden @ weight.T`` of the same bf16 operands.  (2) The select step: the
oracle (``oracle/select_oracle.py``, pinned to the reference's fixtures) run
on exactly those logits must give the same sampled ids, PMI and committed
tokens, with the same near-tie certification as the unfused kernels.  The
sampling chain is the fused path's: temperature, repetition penalty and
Gumbel-max (no top-k / top-p / min-p)."""
import pytest
import torch

from oracle import select_oracle as O
from tests.parity_util import compare
from yapd_b200 import _native as N
from yapd_b200 import select as S
from yapd_b200.workloads import make_config

pytestmark = pytest.mark.gpu


def fused_inputs(seed, B, L=32, masked="all", commit_frac=0.0, explicit=True, rep=None, temperature=None,
                 history=True):
    inp = make_config(4, seed=seed, B=B, L=L, masked=masked, commit_frac=commit_frac, explicit_noise=explicit,
                      lmhead_logits=False)
    inp.top_k = torch.zeros(B, dtype=torch.int32)
    inp.top_p = torch.ones(B)
    inp.min_p = torch.zeros(B)
    if rep is not None:
        inp.rep_penalty = rep.float()
    if temperature is not None:
        inp.temperature = temperature.float()
    if not history:
        inp.history = None
    H = inp.meta["hidden"].view(B, 2, L, -1)
    W = inp.meta["weight"]
    return inp, H, W


def run_fused(inp, H, W, *, noise="explicit", seed=0, offset=0, dense=True, dump=True, **kw):
    dev = torch.device("cuda")
    B, L, V = inp.B, inp.L, inp.V
    lo = torch.empty(B, 2, L, V, dtype=torch.float32, device=dev) if dump else None
    nk = {}
    if noise == "explicit":
        nk = dict(gumbel_tok=inp.gumbel_tok.to(dev), gumbel_pos=inp.gumbel_pos.to(dev))
    out = S.lmhead_select_step(
        H.to(dev), W.to(dev), inp.xt.to(dev), inp.k_step.to(dev), inp.is_commit.to(dev), inp.log_prior.to(dev),
        inp.sched_t.to(dev), inp.q_t.to(dev), cfg_scale=inp.cfg_scale, mask_id=inp.mask_id, stop_id=inp.stop_id,
        temperature=inp.temperature.to(dev), rep_penalty=inp.rep_penalty.to(dev),
        history=None if inp.history is None else inp.history_bitmap().to(dev), pmi_lambda=inp.pmi_lambda,
        pos_noise=inp.pos_noise, use_quantile=inp.use_quantile, seed=seed, offset=offset, dense=dense,
        logits_out=lo, **nk, **kw)
    torch.cuda.synchronize()
    res = {k: getattr(out, k).cpu() for k in
           ("xt", "sampled", "pmi", "n_unmask", "n_mask_after", "hit_eos", "k_step", "is_commit")}
    return res, (None if lo is None else lo.cpu())


def noise_of(inp, noise, seed, offset):
    if noise == "explicit":
        return inp.gumbel_tok
    gt, _ = O.philox_noise(seed, offset, inp.B, inp.L, inp.V)
    return gt


def check_fused(inp, H, W, *, noise="explicit", seed=0, offset=0, dense=True):
    S.clear_status(lmhead=True)
    gpu, lo = run_fused(inp, H, W, noise=noise, seed=seed, offset=offset, dense=dense)
    assert S.read_status(lmhead=True) == 0
    inp.logits = lo.view(inp.B * 2, inp.L, inp.V)
    orc = O.select_step(inp, noise=noise, seed=seed, offset=offset)
    if dense:
        pos = torch.ones(inp.B, inp.L, dtype=torch.bool)
    else:
        pos = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
        assert bool((gpu["sampled"][~pos] == -1).all())
        assert bool(torch.isnan(gpu["pmi"][~pos]).all())
    rep = {}
    compare(inp, gpu, orc, noise_of(inp, noise, seed, offset), positions=pos, report=rep)
    return gpu, lo, rep


def test_gemm_logits_match_fp64():
    """Every logit of every row, the two tail tokens past 8192 included."""
    inp, H, W = fused_inputs(3, B=8)
    _, lo = run_fused(inp, H, W)
    ref = (H.double().reshape(-1, H.shape[-1]) @ W.double().T).view(inp.B, 2, inp.L, inp.V)
    err = (lo.double() - ref).abs()
    # fp32 accumulation of 1024 bf16 products (|logit| ~ 0.6): a misplaced
    # row, column or K block shows as errors of order one
    assert float(err.max()) < 1e-4, float(err.max())
    assert float(err[..., 8192:].max()) < 1e-4


@pytest.mark.parametrize("noise,dense,masked", [("explicit", True, "all"), ("explicit", False, "ragged"),
                                                ("philox", True, "all"), ("philox", False, "ragged")])
def test_fused_select_parity(noise, dense, masked):
    inp, H, W = fused_inputs(7, B=24, masked=masked, commit_frac=0.2 if not dense else 0.0,
                             explicit=noise == "explicit")
    check_fused(inp, H, W, noise=noise, seed=4242, offset=17, dense=dense)


def test_fused_block_of_16_and_ragged_tile():
    """L = 16 (four requests per 64-position tile) and a batch that leaves the
    last tile partly empty."""
    inp, H, W = fused_inputs(11, B=5, L=16, masked="ragged", explicit=False)
    check_fused(inp, H, W, noise="philox", seed=9, offset=3, dense=False)


def test_fused_no_penalty_and_greedy_rows():
    """Unpenalised rows (the plain argmax rule of server/engine.py:546-550)
    and T = 0 rows (greedy, no noise) next to penalised ones."""
    B = 12
    rep = torch.where(torch.arange(B) % 3 == 0, torch.ones(B), torch.full((B,), 1.3))
    T = torch.where(torch.arange(B) % 4 == 1, torch.zeros(B), torch.full((B,), 0.8))
    inp, H, W = fused_inputs(13, B=B, rep=rep, temperature=T)
    check_fused(inp, H, W, noise="explicit")
    inp, H, W = fused_inputs(14, B=B, rep=rep, temperature=T, history=False, explicit=False)
    check_fused(inp, H, W, noise="philox", seed=5, offset=1)


def test_dump_does_not_change_the_result():
    inp, H, W = fused_inputs(17, B=16, masked="ragged", explicit=False)
    a, _ = run_fused(inp, H, W, noise="philox", seed=1, offset=2, dense=False, dump=True)
    b, _ = run_fused(inp, H, W, noise="philox", seed=1, offset=2, dense=False, dump=False)
    for k in a:
        assert torch.equal(a[k], b[k]) or (k == "pmi" and torch.equal(a[k].nan_to_num(7.0), b[k].nan_to_num(7.0)))


def test_unsupported_penalty_leaves_request_unchanged():
    """A repetition penalty below 1 is not served by the fused path: that
    request is left unsampled (-2) with its state unchanged; the others are
    exact."""
    B = 8
    rep = torch.full((B,), 1.2)
    rep[2] = 0.9
    inp, H, W = fused_inputs(19, B=B, rep=rep, masked="ragged")
    S.clear_status(lmhead=True)
    gpu, lo = run_fused(inp, H, W, dense=False)
    st = S.read_status(lmhead=True)
    assert st & N.YAPD_STATUS_ROWS_SKIPPED
    want2 = (inp.xt[2] == inp.mask_id) & ~inp.is_commit[2]
    assert bool((gpu["sampled"][2][want2] == -2).all())
    assert bool((gpu["sampled"][2][~want2] == -1).all())
    assert torch.equal(gpu["xt"][2], inp.xt[2])
    assert int(gpu["k_step"][2]) == int(inp.k_step[2])
    keep = torch.tensor([b for b in range(B) if b != 2])
    sub = subset(inp, keep, lo[keep].reshape(len(keep) * 2, inp.L, inp.V))
    sub.gumbel_tok, sub.gumbel_pos = inp.gumbel_tok[keep], inp.gumbel_pos[keep]
    orc = O.select_step(sub, noise="explicit")
    pos = (sub.xt == sub.mask_id) & ~sub.is_commit[:, None]
    compare(sub, {k: v[keep] for k, v in gpu.items()}, orc, sub.gumbel_tok, positions=pos)


def test_expired_wait_is_reported_and_contained():
    inp, H, W = fused_inputs(23, B=16, masked="ragged", commit_frac=0.2)
    S.clear_status(lmhead=True)
    gpu, _ = run_fused(inp, H, W, dense=False, dump=False, wait_limit_ns=-1)
    st = S.read_status(lmhead=True)
    assert st & N.YAPD_STATUS_WAIT_TIMEOUT
    want = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
    assert bool((gpu["sampled"][want] == -2).all())
    assert bool((gpu["sampled"][~want] == -1).all())
    assert st & N.YAPD_STATUS_ROWS_SKIPPED
    for b in range(inp.B):
        if bool(want[b].any()):
            assert torch.equal(gpu["xt"][b], inp.xt[b])
            assert int(gpu["k_step"][b]) == int(inp.k_step[b])
    # the next call with the default limit is exact again
    check_fused(inp, H, W, dense=False)


def subset(inp, rows, logits):
    """The inputs of requests ``rows`` of ``inp`` as a batch of their own, with
    the given ``(n*2, L, V)`` logits and the Philox noise the full batch drew
    for them (explicit), for the oracle."""
    import dataclasses
    idx = torch.as_tensor(rows)
    per_req = ("xt", "k_step", "is_commit", "temperature", "top_k", "top_p", "min_p", "rep_penalty")
    kw = {k: getattr(inp, k)[idx] for k in per_req}
    kw["history"] = None if inp.history is None else inp.history[idx]
    return dataclasses.replace(inp, logits=logits, **kw)


def test_full_size_config4():
    """BASELINE configuration 4's shape (B = 512 requests x 2 CFG rows x L =
    32, D = 1024, V = 8194) through the fused kernel, Philox noise: the status
    word stays clear, every position gets a token, and 16 requests spread over
    the batch match the oracle on the logits the epilogue consumed."""
    B = 512
    inp, H, W = fused_inputs(29, B=B, explicit=False)
    S.clear_status(lmhead=True)
    gpu, lo = run_fused(inp, H, W, noise="philox", seed=77, offset=5, dense=True)
    assert S.read_status(lmhead=True) == 0
    s = gpu["sampled"]
    assert bool(((s >= 0) & (s < inp.V)).all())
    pick = torch.linspace(0, B - 1, 16).round().long()
    sub = subset(inp, pick, lo[pick].reshape(len(pick) * 2, inp.L, inp.V))
    sub.gumbel_tok, sub.gumbel_pos = O.philox_noise_rows(77, 5, pick.tolist(), inp.L, inp.V)
    orc = O.select_step(sub, noise="explicit")
    got = {k: v[pick] for k, v in gpu.items()}
    compare(sub, got, orc, sub.gumbel_tok)
