"""Drive the unmodified reference select code on the CPU (fixture generation only).

Imports m8than/yapd's ``server.engine`` / ``server.engine_ar`` /
``chatterbox_flash`` modules from a source checkout, with the un-vendored
``chatterbox`` package stubbed (the select step never touches it), and runs:

* ``FlashEngine._step_gpu`` (``server/engine.py:491-622``) with a stub ``self``
  whose forward returns zeros and whose speech head returns the test logits;
  ``server.engine._gumbel_like`` is replaced by a function returning the
  explicit noise tensors in call order (token noise, then position noise);
* ``TurboEngine._sample`` (``server/engine_ar.py:220-243``) with a stub
  ``self`` and ``_gumbel_like`` returning the vocabulary-indexed noise gathered
  by the top-k indices.

Only ``tests/golden/make_golden.py`` and the CPU test that re-checks the oracle
against a live reference checkout use this module; neither runs on the GPU box.
"""
from __future__ import annotations

import os
import sys
import types
from types import SimpleNamespace

import torch

REF_ROOT = os.environ.get("YAPD_REFERENCE_ROOT", "/root/reference")


def reference_available() -> bool:
    return os.path.isfile(os.path.join(REF_ROOT, "server", "engine.py"))


_MODS = None


def load():
    """Import and return ``(engine, engine_ar, model_mod)`` from the reference."""
    global _MODS
    if _MODS is not None:
        return _MODS
    stub_names = [
        "chatterbox", "chatterbox.models", "chatterbox.models.t3", "chatterbox.models.t3.t3",
        "chatterbox.models.t3.modules", "chatterbox.models.t3.modules.cond_enc",
        "chatterbox.models.t3.modules.t3_config",
    ]
    for name in stub_names:
        if name not in sys.modules:
            sys.modules[name] = types.ModuleType(name)
    sys.modules["chatterbox.models.t3.t3"].T3 = torch.nn.Module
    sys.modules["chatterbox.models.t3.modules.cond_enc"].T3Cond = object
    sys.modules["chatterbox.models.t3.modules.t3_config"].T3Config = object
    if "chatterbox_flash" not in sys.modules:
        pkg = types.ModuleType("chatterbox_flash")
        pkg.__path__ = [os.path.join(REF_ROOT, "chatterbox_flash")]
        sys.modules["chatterbox_flash"] = pkg
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    import chatterbox_flash.model as model_mod  # noqa: E402
    import server.engine as engine  # noqa: E402
    import server.engine_ar as engine_ar  # noqa: E402
    _MODS = (engine, engine_ar, model_mod)
    return _MODS


def run_flash_step(inp, g_tok: torch.Tensor, g_pos: torch.Tensor, temp: float,
                   pos_temp: float = 5.0, tau: float = 0.1):
    """One ``FlashEngine._step_gpu`` on the inputs; returns the reference's
    ``flags``, ``xt_final`` and its updated ``k_step``."""
    engine, _, _ = load()
    B, L, V = inp.B, inp.L, inp.V
    nb = inp.nb
    D = 4
    logits = inp.logits.float()
    cols = L + 64
    self = SimpleNamespace(
        n_branch=nb, BS=L, K=inp.num_steps, temp=temp, tau=tau, cfg=inp.cfg_scale,
        posT=pos_temp, MASK=inp.mask_id, STOP=inp.stop_id, V=V, L=cols, N_max=L,
        dtype=torch.float32,
        xt=inp.xt.clone(), blk_start=torch.zeros(B, dtype=torch.long),
        k_step=inp.k_step.clone(), cache_len=torch.zeros(B, dtype=torch.long),
        n_speech=torch.zeros(B, dtype=torch.long), is_commit=inp.is_commit.clone(),
        shift_ctx=torch.zeros(B * nb, 1, D), sched_t=inp.sched_t.clone(), q_t=inp.q_t.clone(),
        ar16=torch.arange(L), arL=torch.arange(cols), log_prior=inp.log_prior.clone(),
        kc=None, vc=None,
    )
    self.t3 = SimpleNamespace(
        _embed_speech_tokens=lambda x: torch.zeros(*x.shape, D),
        speech_head=lambda h: logits.clone(),
    )
    self.core = SimpleNamespace(
        forward=lambda x, pos, pos2, kc, vc, mask, self_attn_only=False, l_used=None:
        torch.zeros(x.shape[0], x.shape[1], D))
    queue = [g_tok.clone(), g_pos.clone()]

    def fake_gumbel(x):
        g = queue.pop(0)
        assert g.shape == x.shape, (g.shape, x.shape)
        return g

    saved = engine._gumbel_like
    engine._gumbel_like = fake_gumbel
    try:
        flags, xt_final = engine.FlashEngine._step_gpu(self, B, L)
    finally:
        engine._gumbel_like = saved
    assert not queue
    return flags, xt_final, self.k_step


def run_turbo_sample(logits_rows: torch.Tensor, seen: torch.Tensor, G_rows: torch.Tensor,
                     temp: float, top_k: int, top_p: float, rep: float) -> torch.Tensor:
    """``TurboEngine._sample`` on ``(R, V)`` rows with uniform parameters; the
    Gumbel noise is ``G_rows`` indexed by vocabulary id."""
    _, engine_ar, _ = load()
    R, V = logits_rows.shape
    self = SimpleNamespace(temp=temp, top_k=top_k, top_p=top_p, rep_p=rep, V=V)
    x = logits_rows
    if temp > 0 and temp != 1.0:
        x = x / temp
    k = min(top_k, V) if top_k > 0 else V
    _, idx = x.topk(k, dim=-1)

    def fake_gumbel(vals):
        assert vals.shape == idx.shape
        return G_rows.gather(1, idx)

    saved = engine_ar._gumbel_like
    engine_ar._gumbel_like = fake_gumbel
    try:
        out = engine_ar.TurboEngine._sample(self, logits_rows, seen)
    finally:
        engine_ar._gumbel_like = saved
    return out


def reference_guided(inp) -> torch.Tensor:
    """CFG-guided log-probabilities through ``cfg_guidance.apply_zero_text_cfg_from_logits``."""
    load()
    from chatterbox_flash.cfg_guidance import apply_zero_text_cfg_from_logits
    B, L, V = inp.B, inp.L, inp.V
    lc = inp.logits.float().view(B, 2, L, V)
    return apply_zero_text_cfg_from_logits(lc[:, 0], lc[:, 1], inp.cfg_scale)


def forcing_noise(sampled: torch.Tensor, V: int) -> torch.Tensor:
    """Noise that makes ``argmax(guided/T + G)`` return ``sampled`` — used to
    push a filtered sample through ``_step_gpu``'s PMI and unmask code."""
    B, L = sampled.shape
    g = torch.zeros(B, L, V)
    g.scatter_(2, sampled.unsqueeze(-1), 1e30)
    return g


class record_internals:
    """Context manager recording, inside one ``_step_gpu`` call, the token
    argmax result (``sampled``) and the input of the descending argsort
    (``where(is_mask, pmi, -inf)``) — the step's sampled ids and ranked PMI."""

    def __enter__(self):
        self.argmax = []
        self.argsort_in = []
        self._am = torch.Tensor.argmax
        self._as = torch.Tensor.argsort
        rec = self

        def argmax(t, *a, **k):
            r = rec._am(t, *a, **k)
            rec.argmax.append(r.clone())
            return r

        def argsort(t, *a, **k):
            rec.argsort_in.append(t.clone())
            return rec._as(t, *a, **k)

        torch.Tensor.argmax = argmax
        torch.Tensor.argsort = argsort
        return self

    def __exit__(self, *exc):
        torch.Tensor.argmax = self._am
        torch.Tensor.argsort = self._as
        return False
