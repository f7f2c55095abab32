"""GPU parity of the select step against the CPU oracle (and the reference fixtures)."""
import os

import numpy as np
import pytest
import torch

from oracle import select_oracle as O
from tests.golden import cases
from tests.parity_util import compare, run_gpu
from yapd_b200 import _native as N
from yapd_b200.workloads import make_config

pytestmark = pytest.mark.gpu
HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _noise(inp, noise, seed, offset):
    if noise == "explicit":
        return inp.gumbel_tok
    gt, _ = O.philox_noise(seed, offset, inp.B, inp.L, inp.V)
    return gt


def check(inp, noise="explicit", seed=0, offset=0, dense=True, history_as="bitmap", scalar_minp=False):
    gpu = run_gpu(inp, noise=noise, seed=seed, offset=offset, dense=dense, history_as=history_as,
                  scalar_minp=scalar_minp)
    orc = O.select_step(inp, noise=noise, seed=seed, offset=offset)
    if dense:
        pos = torch.ones(inp.B, inp.L, dtype=torch.bool)
    else:
        pos = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
        assert bool((gpu["sampled"][~pos] == -1).all())
        assert bool(torch.isnan(gpu["pmi"][~pos]).all())
    rep = {}
    compare(inp, gpu, orc, _noise(inp, noise, seed, offset), positions=pos, report=rep)
    return gpu, orc, rep


@pytest.mark.parametrize("name", cases.REFERENCE_CASES)
def test_reference_fixture(name):
    # the reference's own outputs, exactly: no near-tie is excused here
    inp = cases.build(name)
    gpu, orc, rep = check(inp)
    assert rep.get("certified", 0) == 0
    fx = dict(np.load(os.path.join(HERE, f"{name}.npz")))
    assert np.array_equal(gpu["sampled"].numpy(), fx["sampled"])
    if "xt_final" in fx:
        assert np.array_equal(gpu["xt"].numpy(), fx["xt_final"])


@pytest.mark.parametrize("config,kw", [
    (0, {}),
    (0, dict(masked="ragged", k_step=2)),
    (1, dict(B=8, masked="ragged")),
    (2, dict(B=24, masked="ragged", commit_frac=0.2)),
    (3, dict(B=24, masked="ragged")),
])
def test_configs_explicit_noise(config, kw):
    inp = make_config(config, seed=5, **kw)
    check(inp)


@pytest.mark.parametrize("config", [0, 1, 2])
def test_sparse_mode(config):
    inp = make_config(config, seed=9, B=8 if config else None, masked="ragged", commit_frac=0.25)
    check(inp, dense=False)


@pytest.mark.parametrize("config", [0, 2, 3])
def test_philox_noise(config):
    inp = make_config(config, seed=13, B=6 if config else None, masked="ragged",
                      explicit_noise=False)
    check(inp, noise="philox", seed=1234 + config, offset=7 * config + 1)


# min-p off everywhere, passed as the scalar: bf16 select steps run on the
# grouped kernel alone (the warp kernel only serves min-p positions)
@pytest.mark.parametrize("noise,dense,masked", [("explicit", True, "all"), ("explicit", False, "ragged"),
                                                ("philox", False, "ragged")])
def test_grouped_route_scalar_min_p(noise, dense, masked):
    inp = make_config(3, seed=17, B=24, masked=masked, commit_frac=0.2,
                      explicit_noise=noise == "explicit")
    check(inp, noise=noise, seed=99, offset=3, dense=dense, scalar_minp=True)


def test_history_as_bytes():
    inp = make_config(2, seed=17, B=8, masked="ragged")
    check(inp, history_as="bytes")


def _uniform(inp, **kv):
    B = inp.B
    for name, val in kv.items():
        dt = torch.int32 if name == "top_k" else torch.float32
        setattr(inp, name if name != "rep" else "rep_penalty", torch.full((B,), val, dtype=dt))
    return inp


@pytest.mark.parametrize("kv", [
    dict(temperature=1.2, top_p=0.99),          # large top-p sets (register bisection path)
    dict(temperature=1.0, top_k=1000, top_p=0.97),
    dict(temperature=0.9, top_k=1),
    dict(temperature=0.9, top_k=8193),
    dict(temperature=0.8, top_p=0.0),            # nothing kept -> top-1
    dict(temperature=0.8, min_p=1.5),            # nothing kept -> top-1
    dict(temperature=0.8, rep=1.3),              # penalty only
    dict(temperature=0.0),                       # greedy
    dict(temperature=-1.0, top_p=0.9),
])
def test_parameter_edges(kv):
    inp = make_config(0, seed=21, B=3, L=8)
    inp = _uniform(inp, top_k=0, top_p=1.0, min_p=0.0, rep=1.0)
    inp = _uniform(inp, **kv)
    check(inp)


@pytest.mark.parametrize("V", [17, 33, 64, 6563, 8194])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_vocab_sizes_and_dtypes(V, dtype):
    inp = make_config(0, seed=V, B=2, L=5, V=V, dtype=dtype, masked="ragged")
    check(inp)


def test_no_cfg_branch():
    inp = make_config(0, seed=31, B=4, L=16)
    inp.logits = inp.logits.view(4, 2, 16, -1)[:, 0].contiguous()
    inp.nb = 1
    inp.cfg_scale = 0.0
    check(inp)


def test_ties_bf16_no_cfg():
    # bf16 logits without CFG: many exact ties among vals; top-k/top-p boundaries fall on ties
    inp = make_config(1, seed=41, B=4, L=8, masked="ragged")
    inp.logits = inp.logits.view(4, 2, 8, -1)[:, 0].contiguous()
    inp.nb = 1
    inp.cfg_scale = 0.0
    inp = _uniform(inp, temperature=1.0, top_k=300, top_p=0.9)
    check(inp)


def test_constant_logits_ties():
    inp = make_config(0, seed=43, B=2, L=4)
    inp.logits = torch.zeros_like(inp.logits)
    inp = _uniform(inp, temperature=1.0, top_k=0, top_p=0.5, min_p=0.0, rep=1.0)
    check(inp)


def test_neg_inf_logits():
    inp = make_config(0, seed=47, B=2, L=6)
    inp.logits[:, :, 100:4000] = float("-inf")
    inp = _uniform(inp, temperature=0.8, top_k=0, top_p=0.95, min_p=0.0, rep=1.0)
    check(inp)


def test_edge_masks_and_commit_rows():
    inp = cases.build("flash_edge_masks")
    inp.is_commit = torch.tensor([False, True, False, True])
    check(inp)
    check(inp, dense=False)


def test_sample_rows_matches_turbo_chain():
    from yapd_b200.select import sample_rows
    g = torch.Generator().manual_seed(3)
    R, V = 64, 6563
    logits = torch.randn(R, V, generator=g) * 2
    seen = torch.rand(R, V, generator=g) < 0.02
    G = O.gumbel_from_uniform(torch.rand(R, V, generator=g))
    T = torch.full((R,), 0.8)
    kk = torch.full((R,), 1000, dtype=torch.int32)
    tp = torch.full((R,), 0.95)
    mp = torch.zeros(R)
    rp = torch.full((R,), 1.2)
    want = O.sample_tokens(logits, T, kk, tp, mp, rp, seen, G, zero_temp="unscaled")
    dev = torch.device("cuda")
    got = sample_rows(logits.to(dev), temperature=T.to(dev), top_k=kk.to(dev), top_p=tp.to(dev),
                      min_p=mp.to(dev), rep_penalty=rp.to(dev), seen=seen.to(dev),
                      gumbel=G.to(dev)).cpu().long()
    assert torch.equal(got, want)


def test_status_word_clear():
    from yapd_b200 import select as S
    inp = make_config(0, seed=1)
    run_gpu(inp)
    assert S.read_status() == 0


@pytest.mark.parametrize("B,L", [(3, 5), (40, 32), (300, 27)])
def test_claimed_schedule_counters_return_to_zero(B, L):
    """The grouped kernel's scheduling counters (workspace bytes 64-79: CTAs
    past the preamble, entries appended, entries claimed, CTAs finished) are
    zero after every call, whether the positions are fewer than the CTAs,
    fill each CTA's own stages, or spill into the claimed list; two calls in
    a row on the same workspace give the oracle's result."""
    from yapd_b200 import select as S
    inp = make_config(3, seed=13, B=B, L=L, V=600, masked="ragged", explicit_noise=False)
    for offset in (0, 1):
        gpu = run_gpu(inp, noise="philox", seed=5, offset=offset, dense=False, scalar_minp=True)
        ws = S.workspace(N.lib().yapd_select_workspace_size(B, L), torch.device("cuda"))
        assert ws[64:80].cpu().view(torch.int32).tolist() == [0, 0, 0, 0]
        assert S.read_status() == 0
        orc = O.select_step(inp, noise="philox", seed=5, offset=offset)
        pos = (inp.xt == inp.mask_id) & ~inp.is_commit[:, None]
        gt, _ = O.philox_noise(5, offset, inp.B, inp.L, inp.V)
        compare(inp, gpu, orc, gt, positions=pos)


@pytest.mark.parametrize("scale", [0.9, 1.1, 1.3, 2.0])
@pytest.mark.parametrize("noise", ["explicit", "philox"])
def test_min_p_band_widths(scale, noise):
    # bf16 CFG rows without boosted tokens: the min-p band of a N(0, scale)
    # row holds roughly 140, 90, 45 and 18 tokens for these scales, so the
    # one-lane, the four-per-lane and the deferred band paths all run
    inp = make_config(1, seed=int(scale * 100), B=6, masked="ragged", explicit_noise=(noise == "explicit"))
    g = torch.Generator().manual_seed(int(scale * 1000))
    inp.logits = (torch.randn(inp.logits.shape, generator=g) * scale).to(inp.logits.dtype)
    inp = _uniform(inp, temperature=0.8, top_k=0, top_p=0.95, min_p=0.05, rep=1.2)
    check(inp, noise=noise, seed=99, offset=3, dense=False)


def test_min_p_wide_bands_many_items():
    # 2560 positions: each CTA holds more items than it has warps, so the
    # wide bands of items that are not a warp's last are resolved in the warp
    inp = make_config(1, seed=77, B=80, masked="all")
    g = torch.Generator().manual_seed(7)
    inp.logits = (torch.randn(inp.logits.shape, generator=g) * 1.1).to(inp.logits.dtype)
    inp = _uniform(inp, temperature=0.8, top_k=0, top_p=0.95, min_p=0.05, rep=1.2)
    check(inp, dense=True)


@pytest.mark.parametrize("noise,masked", [("explicit", "ragged"), ("philox", "all")])
def test_lmhead_logits_config4(noise, masked):
    # configuration 4's logits come from a speech head (hidden ~ N(0,1) times a
    # N(0, 0.02) weight): flat rows (std 0.64) whose min-p bands hold hundreds
    # of tokens, so every position takes the wide-band path
    inp = make_config(4, seed=21, B=4, masked=masked, explicit_noise=(noise == "explicit"))
    check(inp, noise=noise, seed=5, offset=2, dense=(masked == "all"))


@pytest.mark.parametrize("top_p,min_p,noise", [(0.95, 0.05, "explicit"), (0.95, 0.05, "philox"),
                                               (1.0, 0.02, "explicit"), (0.3, 0.05, "explicit")])
def test_lmhead_wide_bands_one_warp_teams(top_p, min_p, noise):
    # 2560 positions, so every CTA holds more items than warps and each
    # position has a warp of its own: bands of hundreds of members take the
    # warp's wide min-p path when top-p cannot cut them (0.95, 1.0) and are
    # deferred when it can (0.3)
    inp = make_config(4, seed=31, B=80, masked="all", explicit_noise=(noise == "explicit"))
    inp = _uniform(inp, temperature=0.8, top_k=0, top_p=top_p, min_p=min_p, rep=1.2)
    check(inp, noise=noise, seed=11, offset=4, dense=True)
