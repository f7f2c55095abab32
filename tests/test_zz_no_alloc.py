"""The no-allocation select step (yapd_select_step_noalloc) against yapd_select_step.

The entry point serves callers that cannot allocate device memory: its scratch
lives in a fixed array inside the library instead of a caller workspace.  It
must give the same outputs as the workspace entry point, on consecutive calls
(the shared array keeps the previous call's contents).  This file is collected
last on purpose.
"""
import ctypes as C

import pytest
import torch

from yapd_b200 import _native as N
from yapd_b200 import select as S
from yapd_b200.workloads import make_config

pytestmark = pytest.mark.gpu


def _args(inp, dev, out, keep):
    """yapd_select_args for `inp` (explicit noise) writing into `out`."""
    nb = inp.nb
    lg = inp.logits.to(dev)
    t = {k: getattr(inp, k).to(dev) for k in ("xt", "k_step", "log_prior", "sched_t", "q_t")}
    ic = inp.is_commit.to(dev)
    gt, gp = inp.gumbel_tok.to(dev), inp.gumbel_pos.to(dev)
    hist = inp.history_bitmap().to(dev)
    keep += [lg, ic, gt, gp, hist, *t.values()]
    a = N.SelectArgs()
    a.B, a.nb, a.L, a.V, a.K = inp.B, nb, inp.L, inp.V, inp.num_steps
    a.mask_id, a.stop_id = inp.mask_id, inp.stop_id
    a.logits_dtype = N.YAPD_DTYPE_BF16 if lg.dtype == torch.bfloat16 else N.YAPD_DTYPE_F32
    a.logits = lg.data_ptr()
    a.stride_req, a.stride_branch, a.stride_pos = lg.stride(0) * nb, lg.stride(0), lg.stride(1)
    a.logits_numel = lg.numel()
    a.xt, a.k_step, a.is_commit = t["xt"].data_ptr(), t["k_step"].data_ptr(), ic.data_ptr()
    a.log_prior, a.sched_t, a.q_t = t["log_prior"].data_ptr(), t["sched_t"].data_ptr(), t["q_t"].data_ptr()
    a.cfg_scale, a.cfg_one_plus, a.pmi_lambda = inp.cfg_scale, float(1.0 + inp.cfg_scale), inp.pmi_lambda
    a.pos_noise, a.use_quantile, a.dense = 1, 1, 0
    a.sampling = S._sampling(inp.B, inp.V, dev, inp.temperature.to(dev), inp.top_k.to(dev),
                             inp.top_p.to(dev), inp.min_p.to(dev), inp.rep_penalty.to(dev), hist,
                             True, keep)
    n = N.Noise()
    n.kind, n.gumbel_tok, n.gt_stride_req, n.gt_stride_pos = N.YAPD_NOISE_EXPLICIT, gt.data_ptr(), gt.stride(0), gt.stride(1)
    n.gumbel_pos = gp.data_ptr()
    a.noise = n
    a.xt_out, a.sampled, a.pmi = out.xt.data_ptr(), out.sampled.data_ptr(), out.pmi.data_ptr()
    a.n_unmask, a.n_mask_after = out.n_unmask.data_ptr(), out.n_mask_after.data_ptr()
    a.hit_eos, a.k_step_out, a.is_commit_out = out.hit_eos.data_ptr(), out.k_step.data_ptr(), out.is_commit.data_ptr()
    return a


def _same(x, y):
    assert torch.equal(x.sampled.cpu(), y.sampled.cpu())
    assert torch.equal(x.xt.cpu(), y.xt.cpu())
    for f in ("n_unmask", "n_mask_after", "hit_eos", "k_step", "is_commit"):
        assert torch.equal(getattr(x, f).cpu(), getattr(y, f).cpu()), f
    px, py = x.pmi.cpu().double(), y.pmi.cpu().double()
    ok = torch.isnan(px) == torch.isnan(py)
    assert bool(ok.all())
    fin = ~torch.isnan(px)
    err = ((px - py).abs() / py.abs().clamp_min(1.0))[fin]
    assert err.numel() == 0 or float(err.max()) <= 1e-5


def test_noalloc_matches_workspace_entry_point():
    dev = torch.device("cuda")
    lib = N.lib()
    for cfg, kw in ((1, dict(B=8, masked="ragged", commit_frac=0.2)), (2, dict(B=8, masked="ragged"))):
        inp = make_config(cfg, seed=3, **kw)
        ref = S.SelectOutputs.empty(inp.B, inp.L, dev)
        keep = []
        a_ref = _args(inp, dev, ref, keep)
        ws = torch.zeros(lib.yapd_select_workspace_size(inp.B, inp.L), dtype=torch.uint8, device=dev)
        a_ref.workspace, a_ref.workspace_bytes = ws.data_ptr(), ws.numel()
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        N.check(lib.yapd_select_step(C.byref(a_ref), stream))
        for _ in range(2):  # two calls in a row share the library's scratch array
            got = S.SelectOutputs.empty(inp.B, inp.L, dev)
            a = _args(inp, dev, got, keep)
            N.check(lib.yapd_select_step_noalloc(C.byref(a), stream))
            torch.cuda.synchronize()
            _same(got, ref)


def test_noalloc_rejects_oversize():
    lib = N.lib()
    a = N.SelectArgs()
    a.B, a.L = N.YAPD_NOALLOC_MAX_POSITIONS // 16 + 1, 16
    assert lib.yapd_select_step_noalloc(C.byref(a), None) == -6
