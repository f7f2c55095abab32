/*
 * yapd_select.h — C ABI of the B200 (sm_100a) block-diffusion select step.
 *
 * One call replaces the select body of Chatterbox-Flash's continuous-batching
 * engine, FlashEngine._step_gpu (m8than/yapd server/engine.py:533-612):
 *   CFG combine of cond/uncond speech logits (server/engine.py:533-540,
 *   chatterbox_flash/cfg_guidance.py:33-47), temperature + Gumbel-max token
 *   sampling (server/engine.py:546-550), the Turbo filter chain top-k / top-p /
 *   repetition penalty (server/engine_ar.py:220-243) plus min-p, prior-
 *   calibrated PMI (server/engine.py:553-558, chatterbox_flash/calibration.py:
 *   39-82, cfg_guidance.py:50-57), position noise, the time-shifted quantile
 *   threshold and rank-based unmask (server/engine.py:559-593), and the
 *   per-request state update (server/engine.py:586-622, with the engine's
 *   token buffer, cache / block offsets and flags when args->engine is set).
 *
 * A second entry point, yapd_sample_rows, is TurboEngine._sample
 * (server/engine_ar.py:220-243): one token per V-wide row, no CFG, no PMI.
 *
 * Conventions: every pointer is a device pointer unless stated; shapes are
 * row-major; the functions enqueue work on `stream` (a cudaStream_t, or NULL
 * for the legacy default stream) and never synchronise.  They allocate no
 * memory: scratch comes from the caller's workspace, which must be zero-filled
 * before its first use (a select step keeps its scheduling counters in the
 * workspace header and leaves them at zero when it ends).  A negative return value
 * is a host-side validation error (nothing was launched); YAPD_OK means the
 * kernels were enqueued.  Device-side conditions (a bounded wait that expired)
 * are recorded in the workspace status word, read by yapd_read_status; a
 * select step whose sampling did not finish for some position leaves that
 * position's sampled id at -2 and its request's state unchanged.
 */
#ifndef YAPD_SELECT_H_
#define YAPD_SELECT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define YAPD_ABI_VERSION 4  /* 4: the workspace must be zero-filled before its first call */

/* Return codes (host-side validation; nothing is launched on error). */
#define YAPD_OK 0
#define YAPD_ERR_NULL_POINTER -1
#define YAPD_ERR_BAD_SHAPE -2
#define YAPD_ERR_BAD_DTYPE -3
#define YAPD_ERR_MISALIGNED -4
#define YAPD_ERR_V_TOO_LARGE -5
#define YAPD_ERR_WORKSPACE -6
#define YAPD_ERR_LAUNCH -7
#define YAPD_ERR_BAD_ARG -8
#define YAPD_ERR_NO_DEVICE -9

/* Device status bits (yapd_read_status). */
#define YAPD_STATUS_WAIT_TIMEOUT 1u   /* a bounded pipeline wait expired */
#define YAPD_STATUS_INTERNAL 2u       /* a kernel invariant check failed */
#define YAPD_STATUS_ROWS_SKIPPED 4u   /* a request's state update was skipped:
                                         some of its positions were not sampled
                                         (their sampled id is left at -2) */
#define YAPD_STATUS_CANDIDATE_OVERFLOW 8u  /* fused head: a position had more
                                         near-maximal tokens than its kept-token
                                         slots (its pick may then be off) */

/* Largest vocabulary one logit row may have (register-resident rows). */
#define YAPD_MAX_V 8208
/* Largest block length (positions per request). */
#define YAPD_MAX_L 32

enum yapd_dtype { YAPD_DTYPE_F32 = 0, YAPD_DTYPE_BF16 = 1 };
enum yapd_history_kind {
  YAPD_HISTORY_NONE = 0,
  YAPD_HISTORY_BITMAP = 1, /* int32 words: bit (v&31) of word (v>>5) */
  YAPD_HISTORY_BYTES = 2   /* one byte (bool) per token, as TurboEngine.seen */
};
enum yapd_noise_kind {
  YAPD_NOISE_PHILOX = 0,  /* in-kernel Philox4x32-10 Gumbel noise */
  YAPD_NOISE_EXPLICIT = 1 /* caller-supplied Gumbel tensors (parity mode) */
};

/* Per-request sampling parameters: a NULL array means "use the scalar". */
typedef struct yapd_sampling {
  const float* temperature;  /* (B,) ; T <= 0: see zero_temp_greedy */
  const int32_t* top_k;      /* (B,) ; <= 0 or >= V: off */
  const float* top_p;        /* (B,) ; >= 1: off */
  const float* min_p;        /* (B,) ; <= 0: off */
  const float* rep_penalty;  /* (B,) ; == 1 or no history: off */
  float temperature_s;
  int32_t top_k_s;
  float top_p_s;
  float min_p_s;
  float rep_penalty_s;
  /* 1: T <= 0 takes the argmax without noise (server/engine.py:549-550).
   * 0: T <= 0 skips the division but still samples (server/engine_ar.py:230). */
  int32_t zero_temp_greedy;
  int32_t history_kind;      /* enum yapd_history_kind */
  const void* history;       /* (B, history_stride) words or bytes */
  int64_t history_stride;    /* in words (bitmap) or bytes (bytes) */
} yapd_sampling;

typedef struct yapd_noise {
  int32_t kind;              /* enum yapd_noise_kind */
  uint64_t seed;             /* Philox key */
  uint64_t offset;           /* Philox counter offset (advance per step) */
  const float* gumbel_tok;   /* explicit: (B, L, V) token noise, strides below */
  int64_t gt_stride_req;     /* elements between requests */
  int64_t gt_stride_pos;     /* elements between positions */
  const float* gumbel_pos;   /* explicit: (B, L) contiguous position noise */
} yapd_noise;

/*
 * FlashEngine's whole-generation buffers (server/engine.py:493-497 gathers a
 * request's block from them, :586-622 writes the step's result back).  With
 * yapd_select_args.engine set, the state update also
 *   - scatters xt_final into xt_full at the request's blk_start,
 *   - advances cache_len and blk_start of the requests that were committing
 *     (by L, clamped to cache_limit / blk_limit as the engine clamps them),
 *   - writes the packed flags the engine reads back with its one host sync
 *     (server/engine.py:614-622, 635).
 * args->xt may then be NULL: the block is read from xt_full at blk_start.
 */
typedef struct yapd_engine_state {
  int64_t* xt_full;          /* (B, xt_stride) all tokens of each request */
  int64_t xt_stride;         /* elements between requests (>= blk_limit + L) */
  int64_t* blk_start;        /* (B,) in / out */
  int64_t* cache_len;        /* (B,) in / out */
  const int64_t* n_speech;   /* (B,) copied into the flags */
  int64_t blk_limit;         /* blk_start clamp: N_max - L */
  int64_t cache_limit;       /* cache_len clamp: L_cache - L */
  int64_t* flags;            /* (B, 6): was_commit, n_mask_after, hit_eos,
                                k_step, blk_start, n_speech (after the step) */
} yapd_engine_state;

/*
 * yapd_select_args — one block-diffusion step over B requests.
 *
 * logits element (request b, branch r, position l, token v) lives at
 *   logits + b*stride_req + r*stride_branch + l*stride_pos + v   (elements),
 * branch 0 = conditional, 1 = unconditional (FlashEngine's interleaving,
 * server/engine.py:397-401, 534); the base must be 16-byte aligned and
 * logits_numel bounds every element the call may read.
 */
typedef struct yapd_select_args {
  int32_t B, nb, L, V, K;       /* nb: 2 with CFG, 1 without */
  int64_t mask_id, stop_id;
  int32_t logits_dtype;         /* enum yapd_dtype */
  const void* logits;
  int64_t stride_req, stride_branch, stride_pos, logits_numel;
  const int64_t* xt;            /* (B, L) block tokens (NULL with engine:
                                   read from engine->xt_full) */
  const int64_t* k_step;        /* (B,) */
  const uint8_t* is_commit;     /* (B,) bool */
  const float* log_prior;       /* (V,) log of the clamped prior */
  const int64_t* sched_t;       /* (K,) count schedule */
  const float* q_t;             /* (K,) quantile table */
  float cfg_scale;              /* w */
  float cfg_one_plus;           /* float(1.0 + w), rounded once on the host */
  float pmi_lambda;             /* prior weight; 1 in the engine */
  int32_t pos_noise;            /* position_temperature > 0 */
  int32_t use_quantile;         /* time_shift_tau > 0 */
  int32_t dense;                /* 1: sample every position (the reference's
                                   dense pass); 0: only masked positions of
                                   non-commit requests */
  yapd_sampling sampling;
  yapd_noise noise;
  /* outputs (all required) */
  int64_t* xt_out;              /* (B, L) xt_final; may alias xt */
  int32_t* sampled;             /* (B, L) sampled ids; -1 where not sampled */
  float* pmi;                   /* (B, L) ranked PMI; NaN where not sampled */
  int32_t* n_unmask;            /* (B,) */
  int32_t* n_mask_after;        /* (B,) */
  uint8_t* hit_eos;             /* (B,) */
  int64_t* k_step_out;          /* (B,) may alias k_step */
  uint8_t* is_commit_out;       /* (B,) may alias is_commit */
  void* workspace;
  size_t workspace_bytes;
  /* optional cudaEvent_t pair recorded on `stream` around the sampling
   * kernel (the step's dominant kernel), for roofline timing; NULL = none */
  void* prof_event_begin;
  void* prof_event_end;
  /* optional engine buffers (NULL: the caller keeps them) */
  const yapd_engine_state* engine;
  /* optional device counter: the step adds the number of positions it
     samples (2 logit rows each with CFG), for throughput accounting */
  int64_t* positions_sampled;
  /* limit of each bounded pipeline wait: 0 = the default 0.5 s; < 0 = every
     pipeline wait gives up at once (for testing the failure path); the final
     drain of in-flight copies always waits up to the default */
  int64_t wait_limit_ns;
  /* quantile interpolation of the unmask threshold: 0 = the engine's
     v_lo + (p - lo) * (v_hi - v_lo) (server/engine.py:567-572); 1 =
     torch.quantile's (torch.lerp, fused multiply-add form), as the offline
     block loop computes it (chatterbox_flash/model.py:284) */
  int32_t quantile_lerp;
} yapd_select_args;

/* Rows for TurboEngine._sample: logits (R, V) with row stride `stride_row`. */
typedef struct yapd_sample_args {
  int32_t R, V;
  int32_t logits_dtype;
  const void* logits;
  int64_t stride_row, logits_numel;
  yapd_sampling sampling;       /* per-row parameter arrays are (R,) */
  yapd_noise noise;             /* explicit token noise is (R, V): gt_stride_req */
  int32_t* sampled;             /* (R,) */
  void* workspace;
  size_t workspace_bytes;
  int64_t wait_limit_ns;        /* as in yapd_select_args */
} yapd_sample_args;

/* ABI version of the loaded library (YAPD_ABI_VERSION). */
int yapd_abi_version(void);

/* Human-readable text for a return code. */
const char* yapd_status_string(int code);

/* Workspace bytes a yapd_select_step call over B x L positions needs. */
size_t yapd_select_workspace_size(int32_t B, int32_t L);

/* Workspace bytes a yapd_sample_rows call over R rows needs. */
size_t yapd_sample_workspace_size(int32_t R);

/* Zero the workspace status word (enqueued on `stream`). */
int yapd_clear_status(void* workspace, void* stream);

/* Copy the workspace status word to *status_out (synchronises `stream`). */
int yapd_read_status(const void* workspace, void* stream, uint32_t* status_out);

/*
 * One select step.  Replaces server/engine.py:533-622 (the select body and
 * state update of FlashEngine._step_gpu, called from FlashEngine.tick at
 * server/engine.py:634); with args->engine set it also writes xt_full,
 * cache_len, blk_start and the flags, so the engine's tick is this call plus
 * its one device-to-host copy.  Two kernel launches: token selection (which
 * also builds the work list and initialises the outputs of unsampled
 * positions), then the per-request state update.
 */
int yapd_select_step(const yapd_select_args* args, void* stream);

/*
 * Token sampling over independent rows.  Replaces TurboEngine._sample
 * (server/engine_ar.py:220-243, called at :336 and :406).
 */
int yapd_sample_rows(const yapd_sample_args* args, void* stream);

/* Positions (B * L) the no-allocation entry point accepts. */
#define YAPD_NOALLOC_MAX_POSITIONS 16384

/*
 * yapd_select_step without a caller workspace, for callers that cannot
 * allocate device memory (no cudaMalloc in their process: a foreign memory
 * pool, an allocation-free serving loop, a sandbox with pre-registered
 * buffers).  It has no counterpart in the reference.  Scratch comes from one
 * fixed array in the library's device memory (about 192 KB per device, held
 * until exit); args->workspace and args->workspace_bytes are ignored.
 * B * L above YAPD_NOALLOC_MAX_POSITIONS returns YAPD_ERR_WORKSPACE.
 * The first call on a device looks up that array's device address, so make
 * it before any stream capture.  All calls share the array: calls whose
 * kernels overlap on the GPU race.  The status word is cleared per call and
 * is not readable through yapd_read_status; a call whose sampling did not
 * finish leaves the affected positions' sampled ids at -2 and their requests'
 * state unchanged, which the caller sees in its own outputs.  Arguments are
 * checked before anything is enqueued.
 */
int yapd_select_step_noalloc(const yapd_select_args* args, void* stream);

/*
 * yapd_lmhead_args — the speech head and the select step in one call.
 *
 * The reference computes logits = speech_head(hidden) with a library GEMM
 * (server/engine.py:517-520; chatterbox_flash/engines/flashinfer.py:1452-1461)
 * and then runs the select step on them.  Here the head runs on the tensor
 * cores and the select step's statistics and Gumbel-max scoring run on its
 * accumulators: the logits are never written to device memory.
 *
 * hidden element (request b, branch r, position l, feature d), bf16, lives at
 *   hidden + b*h_stride_req + r*h_stride_branch + l*h_stride_pos + d
 * (branch 0 = conditional, 1 = unconditional); weight is the (V, D) bf16 head
 * with row stride w_stride.  Strides are elements, multiples of 8; both bases
 * 16-byte aligned; D a multiple of 64.
 *
 * select: the select step's arguments as for yapd_select_step, with these
 * restrictions: nb = 2, L = 16 or 32, no top-k / top-p / min-p (NULL arrays,
 * scalars off), repetition penalty >= 1 (a request with a smaller penalty is
 * left unsampled, its state unchanged), history NONE or BITMAP.  Its logits
 * fields are ignored.  select.workspace holds yapd_lmhead_workspace_size bytes
 * (status word first, as for yapd_select_step).  prof_event_begin /
 * prof_event_end bracket the fused GEMM kernel.
 */
typedef struct yapd_lmhead_args {
  const void* hidden;
  int64_t h_stride_req, h_stride_branch, h_stride_pos, hidden_numel;
  const void* weight;
  int64_t w_stride, weight_numel;
  int32_t D;
  float* logits_out;            /* optional fp32 (B, 2, L, V): the logits the
                                   epilogue consumed (for testing); NULL = none */
  yapd_select_args select;
} yapd_lmhead_args;

/* Workspace bytes a yapd_lmhead_select_step call over B x L positions needs. */
size_t yapd_lmhead_workspace_size(int32_t B, int32_t L);

/* Fused speech head + select step.  A memset of the workspace's publication
 * words, then three kernel launches: the tensor-core head GEMM with the select
 * epilogue, the per-position resolve of the kept tokens, and the per-request
 * state update of yapd_select_step. */
int yapd_lmhead_select_step(const yapd_lmhead_args* args, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* YAPD_SELECT_H_ */
