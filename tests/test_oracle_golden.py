"""The CPU oracle against fixtures produced by the unmodified reference."""
import os

import numpy as np
import pytest
import torch

from oracle import select_oracle as O
from tests.golden import cases

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(HERE, f"{name}.npz")))


@pytest.mark.parametrize("name", cases.REFERENCE_CASES)
def test_oracle_matches_reference_fixture(name):
    fx = load(name)
    inp = cases.build(name)
    assert str(fx["digest"]) == cases.input_digest(inp), "input generator drifted"
    res = O.select_step(inp, noise="explicit")
    assert np.array_equal(res["sampled"].numpy(), fx["sampled"]), "sampled ids differ"
    if "pmi_lambda" in fx:
        np.testing.assert_array_equal(res["pmi"].numpy(), fx["pmi_lambda"])
        return
    is_mask = (inp.xt == inp.mask_id).numpy()
    ranked = np.where(is_mask, res["pmi"].numpy(), -np.inf).astype(np.float32)
    np.testing.assert_array_equal(ranked, fx["pmi_ranked"])
    denoise = ~inp.is_commit.numpy()
    assert np.array_equal(res["xt_final"].numpy(), fx["xt_final"])
    assert np.array_equal(res["k_step_final"].numpy(), fx["k_step"])
    assert np.array_equal(res["is_commit_final"].numpy().astype(np.int64)[~denoise], np.zeros((~denoise).sum()))
    flags = fx["flags"]
    assert np.array_equal(res["n_mask_after"].numpy(), flags[:, 1])
    assert np.array_equal(res["hit_eos"].numpy().astype(np.int64), flags[:, 2])


def test_schedule_known_answers():
    from yapd_b200.workloads import omnivoice_unmask_schedule as s
    assert s(16, 10, 0.5) == [1, 1, 1, 1, 1, 2, 2, 2, 2, 3]
    assert s(16, 4, 0.5) == [2, 3, 5, 6]
    assert s(32, 8, 0.5) == [2, 3, 2, 4, 4, 4, 6, 7]
    assert s(0, 5, 0.5) == [0] * 5 and s(7, 1, 0.5) == [7]
    assert sum(s(13, 6, 0.0)) == 13


def test_quantile_lerp_known_answers():
    # m = 0, 1, 2 and L masked positions; q = 0.5 over 4 masked -> p = 1.5
    xt = torch.tensor([[9, 9, 9, 9], [0, 9, 9, 9], [0, 0, 9, 9], [0, 0, 0, 0]])
    mask = 0
    pmi = torch.tensor([[4., 1., 3., 2.], [5., 1., 2., 3.], [1., 2., 7., 5.], [1., 2., 3., 4.]])
    sampled = torch.full((4, 4), 42)
    res = O.unmask_select(pmi, xt, sampled, torch.zeros(4, dtype=torch.long),
                          torch.zeros(4, dtype=torch.bool), torch.tensor([1, 1]),
                          torch.tensor([0.5, 0.0]), mask_id=mask, stop_id=99,
                          num_steps=2, use_quantile=True)
    # row 0: nothing masked -> tau = nan, n_unmask 0
    assert res["n_unmask"][0] == 0
    # row 1: m=1 (position 0): p=0 -> tau=5 -> n_quant=1 -> unmask position 0
    assert res["n_unmask"][1] == 1 and res["xt_final"][1].tolist() == [42, 9, 9, 9]
    # row 2: masked {0,1} with pmi {1,2}: p=0.5 -> tau=1.5 -> n_quant=1 -> position 1
    assert res["n_unmask"][2] == 1 and res["xt_final"][2].tolist() == [0, 42, 9, 9]
    # row 3: all masked, asc=[1,2,3,4], p=1.5 -> tau=2.5 -> n_quant=2
    assert res["n_unmask"][3] == 2
    assert res["xt_final"][3].tolist() == [0, 0, 42, 42]


def test_top_p_strict_boundary():
    # probs exactly [0.5, 0.25, 0.25]: cum_before = [0, .5, .75]; top_p=0.5 keeps only the first
    g = torch.log(torch.tensor([[0.5, 0.25, 0.25]]))
    G = torch.tensor([[0.0, 100.0, 100.0]])
    one = torch.ones(1)
    s = O.sample_tokens(g, one, torch.zeros(1, dtype=torch.int32), torch.tensor([0.5]),
                        torch.zeros(1), one, None, G)
    assert s.item() == 0
    s = O.sample_tokens(g, one, torch.zeros(1, dtype=torch.int32), torch.tensor([0.5001]),
                        torch.zeros(1), one, None, G)
    assert s.item() == 1


def test_penalty_sign_rule():
    g = torch.tensor([[2.0, -1.0, 1.9]])
    seen = torch.tensor([[True, True, False]])
    one = torch.ones(1)
    # rep 1.2: 2.0 -> 1.667 (< 1.9) so token 2 wins with zero noise
    s = O.sample_tokens(g, one, torch.zeros(1, dtype=torch.int32), one, torch.zeros(1),
                        torch.tensor([1.2]), seen, torch.zeros(1, 3))
    assert s.item() == 2
    # negative values are multiplied: -1 * 1.2 = -1.2 stays below
    g2 = torch.tensor([[-1.0, -1.1, -3.0]])
    s = O.sample_tokens(g2, one, torch.zeros(1, dtype=torch.int32), one, torch.zeros(1),
                        torch.tensor([1.2]), torch.tensor([[True, False, False]]), torch.zeros(1, 3))
    assert s.item() == 1


def test_philox_known_answers():
    """Random123's published Philox4x32-10 known-answer vectors."""
    from oracle.philox import philox4x32_10
    cases = [((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
             ((0xFFFFFFFF,) * 4, (0xFFFFFFFF, 0xFFFFFFFF), (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
             ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
              (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1))]
    for ctr, key, want in cases:
        out = philox4x32_10(np.array([ctr], dtype=np.uint32), key)
        assert tuple(int(x) for x in out[0]) == want


def test_lmhead_workload_shapes():
    # configuration 4: the logits are the bf16 rounding of the fp32 head GEMM
    from yapd_b200 import workloads as WL
    inp = WL.make_config(4, seed=1, B=2)
    h, w = inp.meta["hidden"], inp.meta["weight"]
    assert h.shape == (2 * 2 * 32, WL.LMHEAD_HIDDEN) and w.shape == (WL.V_SPEECH, WL.LMHEAD_HIDDEN)
    assert inp.logits.shape == (4, 32, WL.V_SPEECH) and inp.logits.dtype == torch.bfloat16
    ref = (h.float() @ w.float().T).to(torch.bfloat16).view(4, 32, -1)
    assert torch.equal(inp.logits, ref)
    lazy = WL.make_config(4, seed=1, B=2, lmhead_logits=False)
    assert lazy.logits.shape == inp.logits.shape and lazy.logits.stride() == (0, 0, 0)
    assert torch.equal(lazy.meta["hidden"], h)
