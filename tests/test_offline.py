"""The offline generator's block step (chatterbox_flash/model.py:856-906):
the oracle against fixtures the reference's own _pmi_count_early_step_unmask
produced (CPU), and the batched library call against both (GPU)."""
import os

import numpy as np
import pytest
import torch

from oracle import select_oracle as O
from tests.golden import offline_cases as OC

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _oracle(c):
    return O.offline_block_step(c["logits_c"], c["logits_u"], c["xt"], c["done"], k=c["k"], K=c["K"],
                                sched_k=c["sched"][c["k"]], time_shift_tau=c["time_shift_tau"],
                                prior=c["prior"], cfg_scale=c["cfg_scale"], temperature=c["temperature"],
                                position_temperature=c["position_temperature"], G=c["G"], Gpos=c["Gpos"],
                                mask_id=OC.MASK, stop_id=OC.STOP)


@pytest.mark.parametrize("name", list(OC.CASES))
def test_offline_oracle_matches_reference_fixture(name):
    c = OC.build(name)
    fx = dict(np.load(os.path.join(HERE, f"{name}.npz")))
    xt, done = _oracle(c)
    assert np.array_equal(xt.numpy(), fx["xt"])
    assert np.array_equal(done.numpy(), fx["done"])


@pytest.mark.gpu
@pytest.mark.parametrize("name", list(OC.CASES))
def test_offline_block_step_gpu(name):
    from yapd_b200.offline import block_step
    c = OC.build(name)
    fx = dict(np.load(os.path.join(HERE, f"{name}.npz")))
    dev = torch.device("cuda")
    B, bl, K = c["B"], c["bl"], c["K"]
    # the generator's layout: B conditional rows, then B unconditional rows
    blk = c["logits_c"] if c["logits_u"] is None else torch.cat([c["logits_c"], c["logits_u"]], 0)
    log_prior = c["prior"].clamp_min(1e-8).log()
    xt, done = block_step(blk.to(dev), c["xt"].to(dev), c["done"].to(dev), c["k"], cfg_scale=c["cfg_scale"],
                          temperature=c["temperature"], log_prior=log_prior.to(dev),
                          sched_t=torch.tensor(c["sched"], dtype=torch.int64, device=dev),
                          q_t=torch.tensor(c["q"], dtype=torch.float32, device=dev), mask_id=OC.MASK,
                          stop_id=OC.STOP, position_noise=c["position_temperature"] > 0,
                          use_quantile=c["time_shift_tau"] > 0, gumbel_tok=c["G"].to(dev),
                          gumbel_pos=c["Gpos"].to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(xt.cpu().numpy(), fx["xt"])
    assert np.array_equal(done.cpu().numpy(), fx["done"])
