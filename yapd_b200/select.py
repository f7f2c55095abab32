"""Host-side mirror of the reference's select-step interface.

``select_step`` is one call that replaces the select body and state update of
``FlashEngine._step_gpu`` (m8than/yapd ``server/engine.py:533-612``);
``sample_rows`` replaces ``TurboEngine._sample`` (``server/engine_ar.py:220-243``).
Both run the sm_100a kernels of ``libyapd_select.so`` through its C ABI on the
current torch CUDA stream.  Torch is used only for device memory and streams.

Argument meaning follows the reference: ``logits`` is ``(B*nb, L, V)`` with
conditional row ``b*nb`` and unconditional row ``b*nb+1``
(``server/engine.py:534``); ``xt`` the block tokens with ``MASK`` for masked
positions; ``k_step``/``is_commit`` the per-request step counter and commit
flag; ``log_prior`` the log of the clamped unconditional block prior
(``server/engine.py:363-366``); ``sched_t``/``q_t`` the count schedule and
quantile table (``server/engine.py:355-358``).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from . import _native as N
from .workloads import history_to_bitmap


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _extent(t: torch.Tensor) -> int:
    """Elements from ``t``'s first element to one past its last one."""
    return 1 + sum((s - 1) * st for s, st in zip(t.shape, t.stride()))


def _param(x, B: int, dtype, device, name: str):
    """(pointer, scalar) for a per-request parameter given as scalar or (B,) tensor.

    A 0-dim tensor on the CPU is read as a scalar; one on the device is
    broadcast to ``(B,)`` on the device (reading it would synchronise)."""
    if isinstance(x, torch.Tensor):
        if x.numel() == 1 and x.dim() == 0:
            if not x.is_cuda:
                return None, x.item()
            x = x.expand(B)
        if x.shape != (B,):
            raise ValueError(f"{name} must be a scalar or a ({B},) tensor, got {tuple(x.shape)}")
        x = x.to(device=device, dtype=dtype).contiguous()
        return x, 0
    return None, x


@dataclass
class SelectOutputs:
    xt: torch.Tensor            # (B, L) int64 xt_final
    sampled: torch.Tensor       # (B, L) int32, -1 where nothing was sampled
    pmi: torch.Tensor           # (B, L) float32 ranked PMI, NaN where not sampled
    n_unmask: torch.Tensor      # (B,) int32
    n_mask_after: torch.Tensor  # (B,) int32
    hit_eos: torch.Tensor       # (B,) bool
    k_step: torch.Tensor        # (B,) int64 after the step (commit rows reset to 0)
    is_commit: torch.Tensor     # (B,) bool after the step

    @staticmethod
    def empty(B: int, L: int, device) -> "SelectOutputs":
        return SelectOutputs(
            xt=torch.empty(B, L, dtype=torch.int64, device=device),
            sampled=torch.empty(B, L, dtype=torch.int32, device=device),
            pmi=torch.empty(B, L, dtype=torch.float32, device=device),
            n_unmask=torch.empty(B, dtype=torch.int32, device=device),
            n_mask_after=torch.empty(B, dtype=torch.int32, device=device),
            hit_eos=torch.empty(B, dtype=torch.bool, device=device),
            k_step=torch.empty(B, dtype=torch.int64, device=device),
            is_commit=torch.empty(B, dtype=torch.bool, device=device),
        )


@dataclass
class EngineBuffers:
    """FlashEngine's whole-generation buffers (``server/engine.py:493-497``,
    ``:586-622``) for rows ``[0, B)``: the step scatters its block result into
    ``xt_full`` at ``blk_start``, advances ``cache_len`` / ``blk_start`` of
    committing rows (clamped to ``cache_limit`` / ``blk_limit``) and writes
    ``flags`` ``(B, 6)`` int64 = (was_commit, n_mask_after, hit_eos, k_step,
    blk_start, n_speech)."""
    xt_full: torch.Tensor       # (B, >= blk_limit + L) int64, unit column stride
    blk_start: torch.Tensor     # (B,) int64
    cache_len: torch.Tensor     # (B,) int64
    n_speech: torch.Tensor      # (B,) int64
    flags: torch.Tensor         # (B, 6) int64, contiguous
    blk_limit: int              # N_max - L
    cache_limit: int            # L_cache - L


_WORKSPACES: dict = {}


def workspace(nbytes: int, device) -> torch.Tensor:
    """A zero-initialised, cached byte buffer of at least ``nbytes`` on ``device``
    (status word, work list, PMI inputs).

    One buffer serves every call on the device, so the calls of one device must
    be ordered on one stream (the engine's, ``server/engine.py:268-274``):
    calls on two streams that overlap would share the scratch, and a buffer
    replaced by a larger one is freed in the order of the stream that made the
    replacement.  Callers with several streams pass their own workspace through
    the C ABI (``yapd_select_args.workspace``)."""
    dev = torch.device(device)
    key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=dev)
        _WORKSPACES[key] = ws
    return ws


def _history_args(history, B: int, V: int, device):
    if history is None:
        return N.YAPD_HISTORY_NONE, None, 0
    if history.dtype == torch.bool or history.dtype == torch.uint8:
        if history.shape != (B, V):
            raise ValueError(f"bool history must be ({B}, {V})")
        h = history.to(device).contiguous().view(torch.uint8)
        return N.YAPD_HISTORY_BYTES, h, V
    if history.dtype == torch.int32:
        W = (V + 31) // 32
        if history.dim() != 2 or history.shape[0] != B or history.shape[1] < W:
            raise ValueError(f"bitmap history must be ({B}, >= {W}) int32")
        h = history.to(device).contiguous()
        return N.YAPD_HISTORY_BITMAP, h, h.shape[1]
    raise TypeError("history must be bool/uint8 (B, V) or int32 bitmap (B, ceil(V/32))")


def _sampling(B, V, device, temperature, top_k, top_p, min_p, rep_penalty, history,
              zero_temp_greedy, keep):
    s = N.Sampling()
    t, s.temperature_s = _param(temperature, B, torch.float32, device, "temperature")
    k, s.top_k_s = _param(top_k, B, torch.int32, device, "top_k")
    p, s.top_p_s = _param(top_p, B, torch.float32, device, "top_p")
    m, s.min_p_s = _param(min_p, B, torch.float32, device, "min_p")
    r, s.rep_penalty_s = _param(rep_penalty, B, torch.float32, device, "rep_penalty")
    s.temperature, s.top_k, s.top_p, s.min_p, s.rep_penalty = (
        _ptr(t), _ptr(k), _ptr(p), _ptr(m), _ptr(r))
    s.zero_temp_greedy = 1 if zero_temp_greedy else 0
    kind, h, stride = _history_args(history, B, V, device)
    s.history_kind, s.history, s.history_stride = kind, _ptr(h), stride
    keep.extend([t, k, p, m, r, h])
    return s


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return N.YAPD_DTYPE_F32
    if t.dtype == torch.bfloat16:
        return N.YAPD_DTYPE_BF16
    raise TypeError(f"logits must be float32 or bfloat16, got {t.dtype}")


def _common_args(a, B, nb, L, V, dev, keep, xt, k_step, is_commit, log_prior, sched_t, q_t, *,
                 cfg_scale, mask_id, stop_id, temperature, top_k, top_p, min_p, rep_penalty, history,
                 pmi_lambda, pos_noise, use_quantile, gumbel_tok, gumbel_pos, seed, offset,
                 zero_temp_greedy, dense, out, prof_events, engine, positions_sampled, wait_limit_ns,
                 quantile_lerp) -> SelectOutputs:
    """Every field of ``a`` (a ``yapd_select_args``) except the logits and the
    workspace; the tensors the call needs alive go to ``keep``."""
    K = sched_t.numel()
    xt_c = None if xt is None else xt.to(dev, torch.int64).contiguous()
    ks_c = k_step.to(dev, torch.int64).contiguous()
    ic_c = is_commit.to(dev).contiguous().to(torch.bool)
    lp_c = log_prior.to(dev, torch.float32).contiguous()
    st_c = sched_t.to(dev, torch.int64).contiguous()
    qt_c = q_t.to(dev, torch.float32).contiguous()
    keep += [xt_c, ks_c, ic_c, lp_c, st_c, qt_c]
    if out is None:
        out = SelectOutputs.empty(B, L, dev)
    a.B, a.nb, a.L, a.V, a.K = B, nb, L, V, K
    a.mask_id, a.stop_id = int(mask_id), int(stop_id)
    a.xt, a.k_step, a.is_commit = _ptr(xt_c), ks_c.data_ptr(), ic_c.data_ptr()
    a.log_prior, a.sched_t, a.q_t = lp_c.data_ptr(), st_c.data_ptr(), qt_c.data_ptr()
    a.cfg_scale = float(cfg_scale)
    a.cfg_one_plus = float(1.0 + float(cfg_scale))
    a.pmi_lambda = float(pmi_lambda)
    a.pos_noise = 1 if pos_noise else 0
    a.use_quantile = 1 if use_quantile else 0
    a.dense = 1 if dense else 0
    a.sampling = _sampling(B, V, dev, temperature, top_k, top_p, min_p, rep_penalty, history,
                           zero_temp_greedy, keep)
    n = N.Noise()
    if gumbel_tok is not None:
        gt = gumbel_tok.to(dev, torch.float32)
        if gt.stride(2) != 1:
            gt = gt.contiguous()
        gp = None
        if pos_noise:
            if gumbel_pos is None:
                raise ValueError("explicit noise needs gumbel_pos when pos_noise is on")
            gp = gumbel_pos.to(dev, torch.float32).contiguous()
        keep += [gt, gp]
        n.kind = N.YAPD_NOISE_EXPLICIT
        n.gumbel_tok, n.gt_stride_req, n.gt_stride_pos = gt.data_ptr(), gt.stride(0), gt.stride(1)
        n.gumbel_pos = _ptr(gp)
    else:
        n.kind = N.YAPD_NOISE_PHILOX
    n.seed, n.offset = int(seed) & (2**64 - 1), int(offset) & (2**64 - 1)
    a.noise = n
    a.xt_out, a.sampled, a.pmi = out.xt.data_ptr(), out.sampled.data_ptr(), out.pmi.data_ptr()
    a.n_unmask, a.n_mask_after = out.n_unmask.data_ptr(), out.n_mask_after.data_ptr()
    a.hit_eos, a.k_step_out = out.hit_eos.data_ptr(), out.k_step.data_ptr()
    a.is_commit_out = out.is_commit.data_ptr()
    if prof_events is not None:
        a.prof_event_begin, a.prof_event_end = prof_events[0].cuda_event, prof_events[1].cuda_event
    if engine is not None:
        es = N.EngineState()
        xf = engine.xt_full
        for name, t, shape in (("blk_start", engine.blk_start, (B,)), ("cache_len", engine.cache_len, (B,)),
                               ("n_speech", engine.n_speech, (B,)), ("flags", engine.flags, (B, 6))):
            if t.dtype != torch.int64 or tuple(t.shape) != shape or not t.is_contiguous() or t.device != dev:
                raise ValueError(f"engine.{name} must be a contiguous int64 {shape} tensor on {dev}")
        if xf.dtype != torch.int64 or xf.dim() != 2 or xf.shape[0] < B or xf.stride(1) != 1 or xf.device != dev:
            raise ValueError("engine.xt_full must be an int64 (B, N) tensor with unit column stride")
        if xf.shape[1] < int(engine.blk_limit) + L:
            raise ValueError("engine.xt_full is shorter than blk_limit + L")
        es.xt_full, es.xt_stride = xf.data_ptr(), xf.stride(0)
        es.blk_start, es.cache_len = engine.blk_start.data_ptr(), engine.cache_len.data_ptr()
        es.n_speech, es.flags = engine.n_speech.data_ptr(), engine.flags.data_ptr()
        es.blk_limit, es.cache_limit = int(engine.blk_limit), int(engine.cache_limit)
        keep.append(es)
        a.engine = C.addressof(es)
    a.wait_limit_ns = int(wait_limit_ns)
    a.quantile_lerp = 1 if quantile_lerp else 0
    if positions_sampled is not None:
        if positions_sampled.dtype != torch.int64 or positions_sampled.numel() < 1 or positions_sampled.device != dev:
            raise ValueError("positions_sampled must be an int64 device tensor")
        a.positions_sampled = positions_sampled.data_ptr()
    return out


def select_step(logits: torch.Tensor, xt: torch.Tensor, k_step: torch.Tensor,
                is_commit: torch.Tensor, log_prior: torch.Tensor, sched_t: torch.Tensor,
                q_t: torch.Tensor, *, cfg_scale: float, mask_id: int, stop_id: int,
                temperature=0.6, top_k=0, top_p=1.0, min_p=0.0, rep_penalty=1.0,
                history=None, pmi_lambda: float = 1.0, pos_noise: bool = True,
                use_quantile: bool = True, gumbel_tok: torch.Tensor | None = None,
                gumbel_pos: torch.Tensor | None = None, seed: int = 0, offset: int = 0,
                zero_temp_greedy: bool = True, dense: bool = False,
                out: SelectOutputs | None = None,
                prof_events: tuple | None = None, engine: EngineBuffers | None = None,
                L: int | None = None, positions_sampled: torch.Tensor | None = None,
                wait_limit_ns: int = 0, quantile_lerp: bool = False) -> SelectOutputs:
    """One block-diffusion select step (``server/engine.py:533-622``).

    ``nb`` is 2 when ``cfg_scale > 0`` (conditional + unconditional rows) and 1
    otherwise, as ``FlashEngine.n_branch`` (``server/engine.py:322``).  Noise is
    explicit when ``gumbel_tok`` (``(B, L, V)``) and ``gumbel_pos`` (``(B, L)``)
    are given, else generated in-kernel from ``(seed, offset)``.  With
    ``engine`` the step also writes the engine's token buffer, block / cache
    offsets and flags; ``xt`` may then be None (the block is gathered from
    ``engine.xt_full`` in the kernels, ``L`` giving its length).
    ``positions_sampled``, a one-element int64 device tensor, is incremented
    by the number of positions the step samples.  ``wait_limit_ns`` bounds
    each pipeline wait (0: 0.5 s; negative: every pipeline wait gives up at
    once, for testing the failure path).  ``quantile_lerp`` selects
    torch.quantile's interpolation for the unmask threshold (the offline block
    loop's, ``chatterbox_flash/model.py:284``) instead of the engine's.
    ``logits`` may also be a ``(B, nb, L, V)`` view with any strides and a
    unit last stride (e.g. the offline loop's ``[cond rows; uncond rows]``
    layout seen as ``(2, B, L, V).transpose(0, 1)``).
    """
    if not logits.is_cuda:
        raise ValueError("select_step runs on CUDA tensors only (no CPU fallback)")
    if xt is None:
        if engine is None or L is None:
            raise ValueError("xt=None needs engine buffers and the block length L")
        B = engine.blk_start.shape[0]
    else:
        B, L = xt.shape
    nb = 2 if cfg_scale > 0 else 1
    if logits.dim() == 4:
        if tuple(logits.shape[:3]) != (B, nb, L):
            raise ValueError(f"logits must be ({B}, {nb}, {L}, V), got {tuple(logits.shape)}")
        if logits.stride(3) != 1:
            logits = logits.contiguous()
        strides = (logits.stride(0), logits.stride(1), logits.stride(2))
    else:
        if logits.dim() != 3 or logits.shape[0] != B * nb or logits.shape[1] != L:
            raise ValueError(f"logits must be ({B * nb}, {L}, V), got {tuple(logits.shape)}")
        if logits.stride(2) != 1:
            logits = logits.contiguous()
        strides = (logits.stride(0) * nb, logits.stride(0), logits.stride(1))
    V = logits.shape[-1]
    dev = logits.device
    a = N.SelectArgs()
    a.logits_dtype = _dtype_code(logits)
    a.logits = logits.data_ptr()
    a.stride_req, a.stride_branch, a.stride_pos = strides
    a.logits_numel = _extent(logits)
    keep = []
    out = _common_args(a, B, nb, L, V, dev, keep, xt, k_step, is_commit, log_prior, sched_t, q_t,
                       cfg_scale=cfg_scale, mask_id=mask_id, stop_id=stop_id, temperature=temperature,
                       top_k=top_k, top_p=top_p, min_p=min_p, rep_penalty=rep_penalty, history=history,
                       pmi_lambda=pmi_lambda, pos_noise=pos_noise, use_quantile=use_quantile,
                       gumbel_tok=gumbel_tok, gumbel_pos=gumbel_pos, seed=seed, offset=offset,
                       zero_temp_greedy=zero_temp_greedy, dense=dense, out=out, prof_events=prof_events,
                       engine=engine, positions_sampled=positions_sampled, wait_limit_ns=wait_limit_ns,
                       quantile_lerp=quantile_lerp)
    need = N.lib().yapd_select_workspace_size(B, L)
    ws = workspace(need, dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(dev).cuda_stream
    N.check(N.lib().yapd_select_step(C.byref(a), C.c_void_p(stream)))
    return out


_LM_WORKSPACES: dict = {}


def lm_workspace(nbytes: int, device) -> torch.Tensor:
    """The fused head's cached workspace on ``device`` (status word first),
    separate from ``workspace`` because the two layouts differ; the
    one-stream rule of ``workspace`` holds for it too."""
    dev = torch.device(device)
    key = (dev.type, dev.index if dev.index is not None else torch.cuda.current_device())
    ws = _LM_WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 4096), dtype=torch.uint8, device=dev)
        _LM_WORKSPACES[key] = ws
    return ws


def lmhead_select_step(hidden: torch.Tensor, weight: torch.Tensor, xt: torch.Tensor | None,
                       k_step: torch.Tensor, is_commit: torch.Tensor, log_prior: torch.Tensor,
                       sched_t: torch.Tensor, q_t: torch.Tensor, *, cfg_scale: float, mask_id: int,
                       stop_id: int, temperature=0.6, rep_penalty=1.0, history=None,
                       pmi_lambda: float = 1.0, pos_noise: bool = True, use_quantile: bool = True,
                       gumbel_tok: torch.Tensor | None = None, gumbel_pos: torch.Tensor | None = None,
                       seed: int = 0, offset: int = 0, zero_temp_greedy: bool = True, dense: bool = False,
                       out: SelectOutputs | None = None, prof_events: tuple | None = None,
                       engine: EngineBuffers | None = None, L: int | None = None,
                       positions_sampled: torch.Tensor | None = None, wait_limit_ns: int = 0,
                       quantile_lerp: bool = False, logits_out: torch.Tensor | None = None) -> SelectOutputs:
    """The speech head and the select step in one call: ``logits =
    hidden @ weight.T`` (``server/engine.py:517-520``) on the tensor cores,
    with the select step (``server/engine.py:533-622``) run on the GEMM's
    accumulators, so the logits never reach device memory.

    ``hidden``: bf16 ``(B, 2, L, D)`` (cond rows, then uncond rows per
    request) with a unit last stride and strides that are multiples of 8;
    ``weight``: bf16 ``(V, D)``.  The sampling chain is temperature, repetition
    penalty (``>= 1``; history as a bool ``(B, V)`` tensor, converted to a
    bitmap here, or an int32 bitmap) and Gumbel-max: no top-k, top-p or min-p.
    ``logits_out``, an fp32 ``(B, 2, L, V)`` tensor, receives the logits the
    epilogue consumed (for testing).  Everything else is as in ``select_step``.
    """
    if not hidden.is_cuda:
        raise ValueError("lmhead_select_step runs on CUDA tensors only (no CPU fallback)")
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise TypeError("hidden and weight must be bfloat16")
    if hidden.dim() != 4 or hidden.shape[1] != 2:
        raise ValueError(f"hidden must be (B, 2, L, D), got {tuple(hidden.shape)}")
    B, _, Lh, D = hidden.shape
    if xt is not None and tuple(xt.shape) != (B, Lh):
        raise ValueError(f"xt must be ({B}, {Lh})")
    L = Lh
    if hidden.stride(3) != 1 or any(st % 8 for st in hidden.stride()[:3]):
        hidden = hidden.contiguous()
    if weight.dim() != 2 or weight.shape[1] != D:
        raise ValueError(f"weight must be (V, {D})")
    if weight.stride(1) != 1 or weight.stride(0) % 8:
        weight = weight.contiguous()
    V = weight.shape[0]
    dev = hidden.device
    if history is not None and history.dtype in (torch.bool, torch.uint8):
        history = history_to_bitmap(history.to(dev).bool())
    h = N.LmheadArgs()
    h.hidden = hidden.data_ptr()
    h.h_stride_req, h.h_stride_branch, h.h_stride_pos = hidden.stride(0), hidden.stride(1), hidden.stride(2)
    h.hidden_numel = _extent(hidden)
    h.weight, h.w_stride, h.weight_numel = weight.data_ptr(), weight.stride(0), _extent(weight)
    h.D = D
    if logits_out is not None:
        if logits_out.dtype != torch.float32 or tuple(logits_out.shape) != (B, 2, L, V) or \
                not logits_out.is_contiguous():
            raise ValueError(f"logits_out must be a contiguous float32 ({B}, 2, {L}, {V}) tensor")
        h.logits_out = logits_out.data_ptr()
    keep = [hidden, weight, history]
    out = _common_args(h.select, B, 2, L, V, dev, keep, xt, k_step, is_commit, log_prior, sched_t, q_t,
                       cfg_scale=cfg_scale, mask_id=mask_id, stop_id=stop_id, temperature=temperature,
                       top_k=0, top_p=1.0, min_p=0.0, rep_penalty=rep_penalty, history=history,
                       pmi_lambda=pmi_lambda, pos_noise=pos_noise, use_quantile=use_quantile,
                       gumbel_tok=gumbel_tok, gumbel_pos=gumbel_pos, seed=seed, offset=offset,
                       zero_temp_greedy=zero_temp_greedy, dense=dense, out=out, prof_events=prof_events,
                       engine=engine, positions_sampled=positions_sampled, wait_limit_ns=wait_limit_ns,
                       quantile_lerp=quantile_lerp)
    ws = lm_workspace(N.lib().yapd_lmhead_workspace_size(B, L), dev)
    h.select.workspace, h.select.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(dev).cuda_stream
    N.check(N.lib().yapd_lmhead_select_step(C.byref(h), C.c_void_p(stream)))
    return out


def sample_rows(logits: torch.Tensor, *, temperature=0.8, top_k=0, top_p=1.0, min_p=0.0,
                rep_penalty=1.0, seen=None, gumbel: torch.Tensor | None = None, seed: int = 0,
                offset: int = 0, zero_temp_greedy: bool = False,
                out: torch.Tensor | None = None, wait_limit_ns: int = 0) -> torch.Tensor:
    """One token per row of ``logits`` ``(R, V)`` (``server/engine_ar.py:220-243``).

    ``seen`` is the ``(R, V)`` bool history (``server/engine_ar.py:187``) or an
    int32 bitmap.  ``zero_temp_greedy`` defaults to the Turbo rule (``T <= 0``
    still samples, unscaled).
    """
    if not logits.is_cuda:
        raise ValueError("sample_rows runs on CUDA tensors only (no CPU fallback)")
    if logits.dim() != 2:
        raise ValueError("logits must be (R, V)")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    R, V = logits.shape
    dev = logits.device
    keep = []
    if out is None:
        out = torch.empty(R, dtype=torch.int32, device=dev)
    a = N.SampleArgs()
    a.R, a.V = R, V
    a.logits_dtype = _dtype_code(logits)
    a.logits, a.stride_row, a.logits_numel = logits.data_ptr(), logits.stride(0), _extent(logits)
    a.sampling = _sampling(R, V, dev, temperature, top_k, top_p, min_p, rep_penalty, seen,
                           zero_temp_greedy, keep)
    n = N.Noise()
    if gumbel is not None:
        g = gumbel.to(dev, torch.float32)
        if g.stride(1) != 1:
            g = g.contiguous()
        keep.append(g)
        n.kind, n.gumbel_tok, n.gt_stride_req, n.gt_stride_pos = N.YAPD_NOISE_EXPLICIT, g.data_ptr(), g.stride(0), 0
    else:
        n.kind = N.YAPD_NOISE_PHILOX
    n.seed, n.offset = int(seed) & (2**64 - 1), int(offset) & (2**64 - 1)
    a.noise = n
    a.sampled = out.data_ptr()
    a.wait_limit_ns = int(wait_limit_ns)
    ws = workspace(N.lib().yapd_sample_workspace_size(R), dev)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    stream = torch.cuda.current_stream(dev).cuda_stream
    N.check(N.lib().yapd_sample_rows(C.byref(a), C.c_void_p(stream)))
    return out


def read_status(device=None, lmhead: bool = False) -> int:
    """Device status word of the device's workspace, or with ``lmhead`` of the
    fused head's (synchronises the current stream)."""
    dev = torch.device(device or "cuda")
    ws = lm_workspace(256, dev) if lmhead else workspace(256, dev)
    v = C.c_uint32(0)
    N.check(N.lib().yapd_read_status(C.c_void_p(ws.data_ptr()),
                                     C.c_void_p(torch.cuda.current_stream(dev).cuda_stream),
                                     C.byref(v)))
    return v.value


def clear_status(device=None, lmhead: bool = False) -> None:
    """Zero the status word of the device's workspace, or with ``lmhead`` of the
    fused head's (enqueued on the current stream)."""
    dev = torch.device(device or "cuda")
    ws = lm_workspace(256, dev) if lmhead else workspace(256, dev)
    N.check(N.lib().yapd_clear_status(C.c_void_p(ws.data_ptr()),
                                      C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
