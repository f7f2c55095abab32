// Block-diffusion select step for B200 (sm_100a).
//
// Two kernels, launched on the caller's stream (no host sync, no allocation).
// The sampling kernel runs one CTA per SM.  For the select step every CTA
// first scans the block state (which positions are masked in a denoising
// request), writes its own work-list entries and initialises the outputs of
// the positions it will not sample.  With bf16 logits (wsample_kernel) teams
// of warps then work the positions in min-p band mode: each warp streams its
// share of a position's cond / uncond rows through its own ring of 2 KB
// chunks (cp.async.bulk + mbarrier) and computes maxima, the sums of the
// three softmaxes and the candidate band in one pass; the team merges and its
// first warp resolves the band.  Positions that path does not take, and every
// position with fp32 logits or of yapd_sample_rows (sample_kernel), go to the
// grouped pipeline: groups of warps over a 6-deep ring of staged whole rows,
// two statistics passes and a candidate band (no sort of the vocabulary).
// unmask_kernel then runs one warp per request: position noise, quantile
// threshold, count schedule, rank, unmask and the state update.
//
// Reference semantics: server/engine.py:533-612 and server/engine_ar.py:220-243
// of m8than/yapd (see include/yapd_select.h).  The file is compiled with
// -fmad=false so that every a*b+c the reference rounds twice is rounded twice
// here; contractions that are wanted are written as explicit fmaf.
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>

#include <atomic>
#include <mutex>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "yapd_select.h"
#include "philox.cuh"
#include "select_common.cuh"

namespace yapd {

// ----------------------------------------------------------------- config

template <int NT_, int NG_, int W_, int ELEM_, int NSTAGE_>
struct KCfg {
  static constexpr int NT = NT_;        // compute threads per group (one position at a time)
  static constexpr int NG = NG_;        // groups per CTA
  static constexpr int W = W_;          // elements per 16-byte vector
  static constexpr int ELEM = ELEM_;    // bytes per logit
  static constexpr int NSTAGE = NSTAGE_;
  static constexpr int BAND = NT_;      // candidate band capacity (one thread per element)
  static constexpr int NW = NT / 32;    // warps per group
  static constexpr int NTHREADS = NG * NT + NG * 32;  // groups, then one tail warp per group
  static constexpr int ROW_SLOT = ((YAPD_MAX_V * ELEM + 32 + 127) / 128) * 128;
  static constexpr int STAGE_BYTES = 2 * ROW_SLOT;
  static constexpr bool BF16 = (ELEM == 2);
  static constexpr int KV = ((YAPD_MAX_V + 2 * W) / W + NT - 1) / NT;  // vectors per thread per row (max)
  static_assert(NT % 32 == 0 && NT >= 64, "groups are whole warps");
  static_assert(NSTAGE >= NG, "every group needs a stage");
  // Group g waits on full[s] for items g, g + NG, ...; consecutive phases of
  // one stage must go to the same group, or a wait could be posted two phases
  // ahead of the barrier (a parity wait would then pass at once).
  static_assert(NSTAGE % NG == 0, "the groups must divide the stages");
};
using CfgBF16 = KCfg<224, 2, 8, 2, 6>;
using CfgF32 = KCfg<480, 1, 4, 4, 3>;
// fp32 rows without CFG (the Turbo sampler, yapd_sample_rows): one row per
// group, two groups per CTA; a call holds few rows per SM, so two rows in
// flight beat one wider group
using CfgF32R = KCfg<224, 2, 4, 4, 2>;

// Thread index within its group, and the group index.
template <class C>
__device__ __forceinline__ int gtid() { return (int)(threadIdx.x % C::NT); }
template <class C>
__device__ __forceinline__ int gidx() { return threadIdx.x / C::NT; }

constexpr int64_t kWaitLimitNs = 500ll * 1000ll * 1000ll;  // 0.5 s: default pipeline wait, and every drain

// Parameters of the block-state update (server/engine.py:559-612).
struct UnmaskParams {
  const int64_t* xt;
  const int64_t* k_step;
  const uint8_t* is_commit;
  const int64_t* sched_t;
  const float* q_t;
  const int32_t* sampled;
  const float2* pcu;
  const float* log_prior;
  float pmi_lambda, cfg_w, cfg_1pw;
  int nb;
  float* pmi;
  const float* gumbel_pos;
  int noise_kind;
  uint64_t seed, offset;
  int B, L, K;
  int64_t mask_id, stop_id;
  int pos_noise, use_quantile;
  int quantile_lerp;  // 1: torch.quantile's interpolation (torch.lerp)
  int64_t* xt_out;
  int32_t* n_unmask;
  int32_t* n_mask_after;
  uint8_t* hit_eos;
  int64_t* k_step_out;
  uint8_t* is_commit_out;
  // the engine's whole-generation buffers (server/engine.py:493-497, 586-622),
  // or xt_full == null
  int64_t* xt_full;
  int64_t xt_stride;
  int64_t* blk_start;
  int64_t* cache_len;
  const int64_t* n_speech;
  int64_t blk_limit, cache_limit;
  int64_t* flags;
  uint32_t* status;
};

// Block token l of request b: from the caller's (B, L) block, or gathered
// from the engine's token buffer at the request's block start
// (server/engine.py:495-496).
__device__ __forceinline__ int64_t xt_at(const UnmaskParams& U, int b, int l) {
  return U.xt ? U.xt[b * U.L + l] : U.xt_full[(int64_t)b * U.xt_stride + U.blk_start[b] + l];
}

// Unsigned division by an invariant divisor d >= 1 for dividends below 2^31:
// q = umulhi(x, m) >> sh with l = ceil(log2 d), m = ceil(2^(31 + l) / d),
// sh = l - 1 (Granlund and Montgomery, PLDI 1994; for d >= 2, m < 2^32 and
// the error term stays below 1/d).  d = 1 is the identity.
struct DivU {
  uint32_t m;
  int sh;
  int d;
};
static inline DivU divu_make(int d) {
  DivU r{0u, 0, d};
  if (d <= 1) return r;
  int l = 0;
  while ((1ull << l) < (unsigned long long)d) ++l;
  const unsigned long long num = 1ull << (31 + l);
  r.m = (uint32_t)((num + (unsigned long long)d - 1) / (unsigned long long)d);
  r.sh = l - 1;
  return r;
}
__device__ __forceinline__ int divu(int x, const DivU& f) {
  return f.d <= 1 ? x : (int)(__umulhi((uint32_t)x, f.m) >> f.sh);
}

// Kernel parameters (flattened from the C ABI structs on the host).
struct SampleParams {
  // logits
  const char* logits;
  const char* logits_end;  // one past the last byte the call may read
  int64_t stride_req, stride_branch, stride_pos;
  int B, nb, L, V;
  // work: positions p = b*L + l, listed in work_w (select step)
  int n_identity;  // >0: items are 0..n_identity-1 (no work list)
  // sampling
  const float* temperature;
  const int32_t* top_k;
  const float* top_p;
  const float* min_p;
  const float* rep_penalty;
  float temperature_s, top_p_s, min_p_s, rep_penalty_s;
  int32_t top_k_s;
  int zero_temp_greedy;
  int history_kind;
  const void* history;
  int64_t history_stride;
  // noise
  int noise_kind;
  uint64_t seed, offset;
  const float* gumbel_tok;
  int64_t gt_stride_req, gt_stride_pos;
  // CFG weights
  float cfg_w, cfg_1pw;
  // outputs
  int32_t* sampled;
  float2* pcu;  // softmax(c)[s], softmax(u)[s] of the sampled token (PMI inputs), or null
  uint32_t* status;
  // select step: the CTAs build the work list themselves and initialise the
  // outputs of the positions they do not sample
  int fused;
  int dense;                // every position is sampled
  DivU div_L;               // division by L
  DivU div_grid;            // division by the launch's grid size
  int32_t* work_w;          // work list (each CTA writes its own entries)
  unsigned long long* pos_count;  // optional: += positions sampled this step
  int64_t wait_ns;          // limit of each pipeline wait (drains: kWaitLimitNs)
  // select step: the launch's scheduling counters in the workspace header
  // ([0] CTAs past the preamble, [1] work-list entries appended, [2] entries
  // claimed, [3] CTAs finished); zero between calls (the last CTA to finish
  // clears them)
  uint32_t* sched;
  UnmaskParams U;
};

struct RowGeom {
  const char* src;    // 16-byte aligned copy source
  const char* row;    // element 0 of the row
  uint32_t bytes;     // bulk-copy size (multiple of 16, may be 0)
  int head;           // elements before element 0 in the copy
  int avail;          // elements [0, avail) are inside the copy
};

// The record a group leaves for its tail warp: the position's parameters,
// merged statistics and (when `handed`) its min-p band of at most 32 ids.
struct ItemParams {
  int pos;
  float T, top_p, min_p, rep;
  int top_k;
};

struct Hand {
  // written with the stage's copies (by the warp that issues them)
  ItemParams Q;
  RowGeom gc, gu;    // staged cond / uncond rows
  // written by the group
  float m[3], s[3];  // group maxima (c, u, z2') and sums relative to them
  int n;             // band members found (ids of the first 32 in cv)
  int handed;        // 1: the tail warp resolves the min-p band and writes the outputs;
                     // 2: it finishes a histogram select (the fields below)
  int cv[32];
  // histogram select handed to the tail: band P / band K / kept-token ids,
  // their counts, the counts and masses above and between the bands, and the
  // group's best kept token when the kept set is larger than aid
  int hs_nP, hs_nK, hs_nA, hs_sep, hs_kept;  // hs_sep: 0 no band K, 1 band K in kid, 2 S_k in hs_sk
  float hs_na, hs_ma, hs_mP, hs_nb, hs_mb, hs_sk;
  int pid[32], kid[32], aid[64];
};

template <class C>
__device__ __forceinline__ RowGeom row_geom(const SampleParams& P, int64_t elem_off) {
  RowGeom g;
  const uintptr_t start = reinterpret_cast<uintptr_t>(P.logits) + (uintptr_t)(elem_off * C::ELEM);
  const uintptr_t end = start + (uintptr_t)P.V * C::ELEM;
  const uintptr_t a0 = start & ~(uintptr_t)15;
  uintptr_t a1 = (end + 15) & ~(uintptr_t)15;
  const uintptr_t lim = reinterpret_cast<uintptr_t>(P.logits_end) & ~(uintptr_t)15;
  if (a1 > lim) a1 = lim;
  if (a1 < a0) a1 = a0;
  g.src = reinterpret_cast<const char*>(a0);
  g.row = reinterpret_cast<const char*>(start);
  g.bytes = (uint32_t)(a1 - a0);
  g.head = (int)((start - a0) / C::ELEM);
  const int64_t av = ((int64_t)a1 - (int64_t)start) / C::ELEM;
  g.avail = (int)(av < 0 ? 0 : (av > P.V ? P.V : av));
  return g;
}

__device__ __forceinline__ float param_f(const float* a, float s, int b) { return a ? a[b] : s; }
__device__ __forceinline__ int param_i(const int32_t* a, int s, int b) { return a ? a[b] : s; }

// Repetition penalty of server/engine_ar.py:240: v>0 ? v/r : v*r.
__device__ __forceinline__ float penalize(float v, float rep, float rrep) {
  return v > 0.0f ? div_rn(v, rep, rrep) : __fmul_rn(v, rep);
}

// Composite sort key: key descending, then vocabulary id ascending.
__device__ __forceinline__ unsigned long long cand_key(float key, int v) {
  return ((unsigned long long)ord_key(key) << 32) | (uint32_t)(0x7fffffff - v);
}
__device__ __forceinline__ int cand_id(unsigned long long c) { return 0x7fffffff - (int)(uint32_t)c; }
__device__ __forceinline__ float cand_val(unsigned long long c) { return ord_key_inv((uint32_t)(c >> 32)); }

// Shared memory layout.
template <class C>
struct Smem;
template <class C>
struct KSmem;
constexpr int kHistBins = 512;  // bins of the histogram bracket
constexpr int kKqPerWarp = 96;  // kept_pass queue: 32 lanes x at most 3 Philox blocks per vector

template <class C>
__device__ __forceinline__ float load_elem_global(const char* row, int v) {
  if constexpr (C::BF16) {
    const unsigned short h = __ldg(reinterpret_cast<const unsigned short*>(row) + v);
    return __uint_as_float((uint32_t)h << 16);
  } else {
    return __ldg(reinterpret_cast<const float*>(row) + v);
  }
}

template <class C>
__device__ __forceinline__ float load_elem_smem(const unsigned char* s, const RowGeom& g, int v) {
  if (v >= g.avail) return load_elem_global<C>(g.row, v);
  const uint32_t a = smem_u32(s) + (uint32_t)(v + g.head) * C::ELEM;
  if constexpr (C::BF16) {
    unsigned short h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(a));
    return __uint_as_float((uint32_t)h << 16);
  } else {
    float f;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(f) : "r"(a));
    return f;
  }
}

// ------------------------------------------------------------ streaming geometry
//
// The staged copy of a row starts `head` elements before element 0.  Vectors
// (16 bytes) j in [j0, j1) lie wholly inside [0, avail) of both rows (the cond
// and uncond copies share their head); the remaining elements, at most a few
// per row end, are "scalar" elements e in [0, nscal) with id scalar_v(e).
// When the two rows have different heads every element is scalar.
struct Span {
  int j0, j1;  // interior vectors
  int head;    // elements before element 0 in vector 0
  int nlo;     // scalar elements [0, nlo) ...
  int hi0;     // ... and [hi0, V)
  int nscal;
};

__device__ __forceinline__ int scalar_v(const Span& S, int e) { return e < S.nlo ? e : S.hi0 + (e - S.nlo); }

// Element i of a 16-byte vector.
template <class C>
__device__ __forceinline__ float velem(const uint4& q, int i) {
  const uint32_t w = (i / (C::BF16 ? 2 : 1)) == 0 ? q.x : (i / (C::BF16 ? 2 : 1)) == 1 ? q.y
                   : (i / (C::BF16 ? 2 : 1)) == 2 ? q.z : q.w;
  if constexpr (C::BF16) return (i & 1) ? bf16hi(w) : bf16lo(w);
  else return __uint_as_float(w);
}

// 16-byte load from the staged rows (explicitly shared-space: the ring is
// reached through pointers the compiler cannot always classify).
__device__ __forceinline__ uint4 lds128(const unsigned char* p) {
  uint4 r;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "r"(smem_u32(p)));
  return r;
}

__device__ __forceinline__ uint32_t bmax2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bmin2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("min.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Total order used to rank PMI: NaN above +inf (torch's sort order).
__device__ __forceinline__ uint32_t rank_key(float f) {
  return (f != f) ? 0xffffffffu : ord_key(f);
}

// Block-state update of request b by one warp: server/engine.py:559-612.
// Only the positions sampled this step (every position in dense mode, else
// the masked positions of a denoising request) use `sampled` and `pcu`.
__device__ __forceinline__ void unmask_request(const UnmaskParams& U, int dense, int b) {
  const int lane = threadIdx.x & 31;
  const int L = U.L, K = U.K;
  const bool in = lane < L;
  const int p = b * L + lane;
  // every load that does not depend on another goes out first (lanes past L
  // read the request's first position and ignore it)
  const int pc = in ? p : b * L;
  const int64_t xr = xt_at(U, b, in ? lane : 0);
  const int64_t bs = U.xt_full ? U.blk_start[b] : 0;
  const uint8_t cm = U.is_commit[b];
  const int64_t ks = U.k_step[b];
  const int sraw = U.sampled[pc];   // -1 where not sampled this step
  const float2 pr = U.pcu[pc];      // read only where sampled
  const int64_t x = in ? xr : 0;
  const bool is_mask = in && x == U.mask_id;
  const bool commit = cm != 0;
  const bool denoise = !commit;
  int kc = (int)(ks < (int64_t)(K - 1) ? ks : (int64_t)(K - 1));
  if (kc < 0) kc = 0;
  // PMI of the sampled token (server/engine.py:553-558, calibration.py:58-60)
  // and the position noise on masked positions (server/engine.py:559-561)
  float gn = 0.f;
  if (is_mask && U.pos_noise)
    gn = (U.noise_kind == YAPD_NOISE_EXPLICIT) ? U.gumbel_pos[p]
                                                : philox_position_gumbel(U.seed, U.offset, (uint32_t)p);
  float pm = 0.f;
  const bool want = in && (dense || (!commit && x == U.mask_id));
  // a masked position of a denoising request that this step had to sample but
  // did not (its id left at -2 after an expired wait): the request keeps its
  // state (commit rows do not use their samples)
  const bool skip = __any_sync(0xffffffffu, want && !commit && sraw < 0);
  const int smp = (want && !skip && sraw >= 0) ? sraw : -1;
  if (smp >= 0) {
    const float lpl = __fmul_rn(U.pmi_lambda, __ldg(U.log_prior + smp));
    pm = __fsub_rn(logf(fmaxf(pr.x, 1e-8f)), lpl);
    if (U.nb == 2) {
      const float pmi_u = __fsub_rn(logf(fmaxf(pr.y, 1e-8f)), lpl);
      pm = __fsub_rn(__fmul_rn(U.cfg_1pw, pm), __fmul_rn(U.cfg_w, pmi_u));
    }
  }
  if (is_mask && U.pos_noise) pm = __fadd_rn(pm, gn);
  const unsigned mbal = __ballot_sync(0xffffffffu, is_mask);
  const int m = __popc(mbal);
  // ascending sort of masked PMI (+inf elsewhere), engine.py:566
  const uint32_t ak = is_mask ? rank_key(pm) : ord_key(__int_as_float(0x7f800000));
  uint32_t srt = ak;
#pragma unroll
  for (int kk = 2; kk <= 32; kk <<= 1) {
#pragma unroll
    for (int j = kk >> 1; j > 0; j >>= 1) {
      const uint32_t y = __shfl_xor_sync(0xffffffffu, srt, j);
      const bool up = ((lane & kk) == 0);
      const bool lower = ((lane & j) == 0);
      const bool take_min = (up == lower);
      srt = take_min ? min(srt, y) : max(srt, y);
    }
  }
  const float asc = (srt == 0xffffffffu) ? __int_as_float(0x7fc00000) : ord_key_inv(srt);
  // quantile by linear interpolation (engine.py:567-572)
  const float q = U.q_t[kc];
  const float pq = __fmul_rn(q, (float)(m - 1 > 0 ? m - 1 : 0));
  int lo = (int)floorf(pq), hi = (int)ceilf(pq);
  lo = lo < 0 ? 0 : (lo > 31 ? 31 : lo);
  hi = hi < 0 ? 0 : (hi > 31 ? 31 : hi);
  const float v_lo = __shfl_sync(0xffffffffu, asc, lo);
  const float v_hi = __shfl_sync(0xffffffffu, asc, hi);
  const float wq = __fsub_rn(pq, (float)lo), dq = __fsub_rn(v_hi, v_lo);
  float tau;
  if (!U.quantile_lerp) {
    tau = __fadd_rn(v_lo, __fmul_rn(wq, dq));
  } else {
    // torch.quantile (chatterbox_flash/model.py:284) interpolates with
    // torch.lerp: a + w*(b - a) for w < 1/2, else b - (b - a)*(1 - w), each a
    // fused multiply-add
    tau = fabsf(wq) < 0.5f ? __fmaf_rn(wq, dq, v_lo) : __fmaf_rn(-dq, __fsub_rn(1.0f, wq), v_hi);
  }
  int n_quant = __popc(__ballot_sync(0xffffffffu, is_mask && pm >= tau));
  if (!U.use_quantile) n_quant = 0;
  const int64_t sch = U.sched_t[kc];
  const int n_sched = (int)(sch < (int64_t)m ? sch : (int64_t)m);
  int n_un = min(max(n_sched, n_quant), m);
  if (ks >= (int64_t)(K - 1)) n_un = m;
  if (m == 0) n_un = 0;
  // rank among masked positions by PMI descending, ties to the lower position (engine.py:581-584)
  const uint32_t mk = rank_key(pm);
  int rank = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const uint32_t kj = __shfl_sync(0xffffffffu, mk, j);
    const bool mj = (mbal >> j) & 1u;
    rank += (mj && (kj > mk || (kj == mk && j < lane))) ? 1 : 0;
  }
  const bool do_un = is_mask && rank < n_un;
  int64_t xf = x;
  if (denoise && do_un && !skip) xf = (int64_t)U.sampled[p];
  if (in) {
    U.xt_out[p] = xf;
    if (smp >= 0) U.pmi[p] = pm;
    else if (want) U.pmi[p] = __int_as_float(0x7fc00000);
    // server/engine.py:586: the block goes back into the token buffer
    if (U.xt_full) U.xt_full[(int64_t)b * U.xt_stride + bs + lane] = xf;
  }
  const int n_after = __popc(__ballot_sync(0xffffffffu, in && xf == U.mask_id));
  const bool eos = __any_sync(0xffffffffu, in && xf == U.stop_id);
  if (lane == 0) {
    const int64_t k_new = (denoise && !skip) ? ks + 1 : ks;
    const int64_t k_fin = commit ? 0 : k_new;
    const bool to_commit = denoise && !skip && !eos && (n_after == 0 || k_fin >= (int64_t)K);
    if (skip) atomicOr(U.status, (unsigned)YAPD_STATUS_ROWS_SKIPPED);
    U.n_unmask[b] = (denoise && !skip) ? n_un : 0;
    U.n_mask_after[b] = n_after;
    U.hit_eos[b] = eos ? 1 : 0;
    U.k_step_out[b] = k_fin;
    U.is_commit_out[b] = to_commit ? 1 : 0;
    if (U.xt_full) {
      // commit rows move to the next block (server/engine.py:597-603, the
      // engine's clamps keep inert rows in range) and the packed flags
      // (:614-622) for the engine's one host sync
      const int64_t cl = U.cache_len[b];
      const int64_t cl2 = commit ? min(cl + (int64_t)L, U.cache_limit) : cl;
      const int64_t bs2 = commit ? min(bs + (int64_t)L, U.blk_limit) : bs;
      U.cache_len[b] = cl2;
      U.blk_start[b] = bs2;
      int64_t* f = U.flags + (int64_t)b * 6;
      f[0] = commit ? 1 : 0;
      f[1] = n_after;
      f[2] = eos ? 1 : 0;
      f[3] = k_fin;
      f[4] = bs2;
      f[5] = U.n_speech[b];
    }
  }
}

// One warp per request: the block-state update after the sample kernel.
__global__ void unmask_kernel(const __grid_constant__ UnmaskParams U, int dense) {
  // launched as a programmatic dependent of the sampling kernel: its CTAs
  // may be resident before that kernel ends, and wait here until it has
  // finished and its writes are visible (no effect on an ordinary launch)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b < U.B) unmask_request(U, dense, b);
}

// Sampling parameters of the first RCAP requests, kept on chip by the
// preamble of the warp kernel.
constexpr int kReqCap = 512;
struct ReqTable {
  float T[kReqCap], top_p[kReqCap], min_p[kReqCap], rep[kReqCap];
  int top_k[kReqCap];
};

__device__ __forceinline__ ItemParams load_params(const SampleParams& P, int pos) {
  ItemParams q;
  const int b = pos / P.L;
  q.pos = pos;
  q.T = param_f(P.temperature, P.temperature_s, b);
  q.top_k = param_i(P.top_k, P.top_k_s, b);
  q.top_p = param_f(P.top_p, P.top_p_s, b);
  q.min_p = param_f(P.min_p, P.min_p_s, b);
  q.rep = param_f(P.rep_penalty, P.rep_penalty_s, b);
  return q;
}

// The request table: every thread loads the parameters of requests
// threadIdx.x + k * blockDim.x (the first kReqCap).
__device__ __forceinline__ void load_req_table(const SampleParams& P, ReqTable& rt) {
  const int nb = min(P.B, kReqCap);
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    rt.T[b] = param_f(P.temperature, P.temperature_s, b);
    rt.top_k[b] = param_i(P.top_k, P.top_k_s, b);
    rt.top_p[b] = param_f(P.top_p, P.top_p_s, b);
    rt.min_p[b] = param_f(P.min_p, P.min_p_s, b);
    rt.rep[b] = param_f(P.rep_penalty, P.rep_penalty_s, b);
  }
}

// Select step, preamble run by every CTA: scan the block state (warps own
// contiguous spans of positions), count the sampled positions and write the
// work-list entries this CTA will process (entries blockIdx + k*gridDim);
// initialise the outputs of the unsampled positions p == blockIdx (mod
// gridDim) (sampled -1, pmi NaN).  Returns the number of sampled positions.
// With `rt`, the request table is loaded alongside the first scan loads and
// the positions of the CTA's first `cap` items go to items_pos[].
__device__ int cta_prepare(const SampleParams& P, int* scan, ReqTable* rt = nullptr, int* items_pos = nullptr,
                           int cap = 0) {
  const UnmaskParams& U = P.U;
  const int total = U.B * U.L;
  const int nwarp = blockDim.x >> 5;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int grid = (int)gridDim.x, me = (int)blockIdx.x;
  // warp w owns positions [w0, w1), read 32 per round, kR rounds per chunk;
  // every load is issued (clamped in range) before any of them is used
  constexpr int kR = 8;
  const int span = (((total + nwarp - 1) / nwarp) + 31) & ~31;
  const int w0 = min(w * span, total), w1 = min(w0 + span, total);
  const bool one_chunk = span <= kR * 32;
  auto chunk = [&](int c0, unsigned (&m)[kR], bool with_table) {
    int64_t xv[kR];
    uint8_t cv[kR];
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int pc = min(c0 + r * 32 + lane, total - 1);
      const int bq = divu(pc, P.div_L);
      xv[r] = xt_at(U, bq, pc - bq * U.L);
      cv[r] = U.is_commit[bq];
    }
    // the table loads go out while the scan loads are in flight
    if (with_table) load_req_table(P, *rt);
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int p = c0 + r * 32 + lane;
      m[r] = __ballot_sync(0xffffffffu, p < w1 && (P.dense || (cv[r] == 0 && xv[r] == U.mask_id)));
    }
  };
  unsigned masks[kR];
  int cnt = 0;
  for (int c0 = w0; c0 < w1; c0 += kR * 32) {
    chunk(c0, masks, rt != nullptr && c0 == w0);
#pragma unroll
    for (int r = 0; r < kR; ++r) cnt += __popc(masks[r]);
  }
  if (rt != nullptr && w0 >= w1) load_req_table(P, *rt);
  if (lane == 0) scan[w] = cnt;
  __syncthreads();
  int base = 0, tot = 0;
  for (int q = 0; q < nwarp; ++q) {
    const int c = scan[q];
    base += q < w ? c : 0;
    tot += c;
  }
  if (P.pos_count && blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(P.pos_count, (unsigned long long)tot);
  // this CTA's entries: global indices me + k*grid (the k-th item) and, for
  // the output initialisation, positions me + j*grid; both stride by grid,
  // so each round of 32 meets few of them (warp-uniform loops)
  int nxt = base <= me ? me : me + divu(base - me + grid - 1, P.div_grid) * grid;
  int np = w0 <= me ? me : me + divu(w0 - me + grid - 1, P.div_grid) * grid;
  for (int c0 = w0; c0 < w1; c0 += kR * 32) {
    if (!one_chunk) chunk(c0, masks, false);
#pragma unroll
    for (int r = 0; r < kR; ++r) {
      const int p0 = c0 + r * 32;
      const int cr = __popc(masks[r]);
      while (nxt < base + cr) {
        const int ln = (int)__fns(masks[r], 0u, nxt - base + 1);
        if (lane == ln) {
          P.work_w[nxt] = p0 + lane;
          P.sampled[p0 + lane] = -2;  // until this CTA samples it
          const int qi = divu(nxt - me, P.div_grid);
          if (qi < cap) items_pos[qi] = p0 + lane;
        }
        nxt += grid;
      }
      while (np < min(p0 + 32, w1)) {
        if (lane == np - p0 && !((masks[r] >> lane) & 1u)) {
          P.sampled[np] = -1;
          U.pmi[np] = __int_as_float(0x7fc00000);
        }
        np += grid;
      }
      base += cr;
    }
  }
  __syncthreads();
  return tot;
}

// Select step, preamble of the grouped kernel's claimed schedule: CTA c
// scans only its share of the positions, [c * span, (c + 1) * span), marks
// the sampled ones -2 (until they are sampled) and initialises the outputs of
// the others (sampled -1, pmi NaN), keeps its first `cap` sampled positions
// for itself (own[], in position order) and appends the rest to the launch's
// work list (one reservation on sched[1] per round of blockDim positions).
// Returns the number of own positions.
__device__ int cta_prepare_share(const SampleParams& P, int* own, int cap, int* scan) {
  const UnmaskParams& U = P.U;
  const int total = U.B * U.L;
  const int grid = (int)gridDim.x;
  const int span = (total + grid - 1) / grid;
  const int p0 = min((int)blockIdx.x * span, total), p1 = min(p0 + span, total);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nwarp = blockDim.x >> 5;
  int done = 0;
  for (int r0 = p0; r0 < p1; r0 += blockDim.x) {
    const int p = r0 + (int)threadIdx.x;
    bool smp = false;
    if (p < p1) {
      const int b = divu(p, P.div_L);
      smp = P.dense || (U.is_commit[b] == 0 && xt_at(U, b, p - b * U.L) == U.mask_id);
      if (smp) {
        P.sampled[p] = -2;
      } else {
        P.sampled[p] = -1;
        U.pmi[p] = __int_as_float(0x7fc00000);
      }
    }
    const unsigned bal = __ballot_sync(0xffffffffu, smp);
    if (lane == 0) scan[w] = __popc(bal);
    __syncthreads();
    int before = 0, cnt = 0;
    for (int q = 0; q < nwarp; ++q) {
      const int c = scan[q];
      before += q < w ? c : 0;
      cnt += c;
    }
    const int rank = done + before + __popc(bal & ((1u << lane) - 1u));  // among the CTA's sampled positions
    const int first_app = max(done, cap);                                // first rank appended in this pass
    const int n_app = max(0, done + cnt - first_app);
    if (threadIdx.x == 0 && n_app > 0) scan[nwarp] = (int)atomicAdd(P.sched + 1, (unsigned)n_app);
    __syncthreads();
    if (smp) {
      if (rank < cap) own[rank] = p;
      else P.work_w[scan[nwarp] + (rank - first_app)] = p;
    }
    done += cnt;
    __syncthreads();
  }
  if (P.pos_count && threadIdx.x == 0 && done > 0) atomicAdd(P.pos_count, (unsigned long long)done);
  return min(done, cap);
}

// ------------------------------------------------------------ sample kernel

// Issue the copies of position Q.pos into `stage` and record its parameters
// and row geometry for the group (one thread).
template <class C>
__device__ __forceinline__ void issue_item(const SampleParams& P, KSmem<C>& ks, int stage, const ItemParams& Q) {
  const int pos = Q.pos;
  const int b = pos / P.L, l = pos - b * P.L;
  const int64_t base = (int64_t)b * P.stride_req + (int64_t)l * P.stride_pos;
  const RowGeom gc = row_geom<C>(P, base);
  uint32_t bytes = gc.bytes;
  RowGeom gu = gc;
  if (P.nb == 2) {
    gu = row_geom<C>(P, base + P.stride_branch);
    bytes += gu.bytes;
  }
  Hand& h = ks.hand[stage];
  h.Q = Q;
  h.gc = gc;
  h.gu = gu;
  mbar_arrive_expect_tx(&ks.full[stage], bytes);
  if (gc.bytes) bulk_g2s(ks.stage[stage], gc.src, gc.bytes, &ks.full[stage]);
  if (P.nb == 2 && gu.bytes) bulk_g2s(ks.stage[stage] + C::ROW_SLOT, gu.src, gu.bytes, &ks.full[stage]);
}

template <class C>
__device__ __forceinline__ int item_pos(const SampleParams& P, int idx) {
  return P.n_identity > 0 ? idx : P.work_w[idx];
}

// Barrier over the warps of this thread's group (named barrier 1 + group).
template <class C>
__device__ __forceinline__ void csync() {
  named_sync(1 + gidx<C>(), C::NT);
}

// OR of a predicate over the group (one barrier).
template <class C>
__device__ __forceinline__ bool csync_or(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(1 + gidx<C>()), "n"(C::NT)
      : "memory");
  return r != 0;
}

// ------------------------------------------------------------ per-position core
//
// Each position is worked by one group of warps from its staged rows in shared
// memory.  Hot path (streaming 16-byte vectors): per-thread maxima, then the
// sums of exp(x - max) and of 2^(z2 - ref) against per-thread references, with
// z2 = log2(e) * (guided / T) - const computed with two FMAs from the
// cond/uncond logits, merged across the group by rescaling; then the min-p
// candidate band.  Cold paths (unfiltered argmax, top-k / top-p bracketing,
// massive ties, NaN rows) recompute z2 element by element in rolled loops.
// Every decision that the reference's float rounding can flip is taken on
// exact values recomputed with the reference's op order (exact_val).

struct PosCtx {
  float mc, mu;   // row maxima
  float lc, lu;   // log of sum(exp(x - max)) per row
  float Sc, Su;   // the sums
  float zmax, S;  // max of z2 and sum of 2^(z2 - zmax)
  float A2, B2, K2;  // z2 = A2*c - B2*u + K2
  float Kval;     // guided/T ~= z2*ln2 + Kval
  float T, rT;
  bool scale, cfg;
};

constexpr float kLn2 = 0.69314718055994531f;
constexpr float kBig = 3.0e38f;

// Bound on |z2 - log2(e)*vals - const| (float rounding of the FMA form against
// the reference's op sequence), with a wide safety factor.
__device__ __forceinline__ float zmargin(float z) { return 2e-4f + 2e-5f * fabsf(z); }

template <class C>
struct RowRef {
  const unsigned char* sc;
  const unsigned char* su;
  RowGeom gc, gu;
};

// guided / T exactly as the reference rounds it (server/engine.py:536-538,
// :548), from the token's cond / uncond logits.
__device__ __forceinline__ float exact_val_cu(const SampleParams& P, const PosCtx& X, float c, float u) {
  float g;
  if (X.cfg) {
    const float lsc = __fsub_rn(__fsub_rn(c, X.mc), X.lc);
    const float lsu = __fsub_rn(__fsub_rn(u, X.mu), X.lu);
    g = __fadd_rn(lsc, __fmul_rn(P.cfg_w, __fsub_rn(lsc, lsu)));
  } else {
    g = c;
  }
  return X.scale ? div_rn(g, X.T, X.rT) : g;
}

template <class C>
__device__ __forceinline__ float exact_val(const SampleParams& P, const PosCtx& X, const RowRef<C>& R, int v) {
  const float c = load_elem_smem<C>(R.sc, R.gc, v);
  const float u = X.cfg ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
  return exact_val_cu(P, X, c, u);
}

__device__ __forceinline__ float z2_of(const PosCtx& X, float c, float u) {
  return X.cfg ? __fmaf_rn(c, X.A2, __fmaf_rn(u, -X.B2, X.K2)) : __fmaf_rn(c, X.A2, X.K2);
}

// The register pass's z2 for token v, recomputed from the staged rows.
template <class C>
__device__ __forceinline__ float z2_smem(const PosCtx& X, const RowRef<C>& R, int v) {
  const float c = load_elem_smem<C>(R.sc, R.gc, v);
  const float u = X.cfg ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
  return z2_of(X, c, u);
}

template <class C, bool CFG>
__device__ __forceinline__ Span make_span(const RowRef<C>& R, int V);

// Every element of the staged rows with its z2 (z2_smem's value): the 16-byte
// vectors first (one thread per vector), then the elements of the partial
// vectors at the row ends.
template <class C, class F>
__device__ __forceinline__ void for_each_z(const PosCtx& X, const RowRef<C>& R, int V, F&& f) {
  const int tid = gtid<C>();
  const Span S = X.cfg ? make_span<C, true>(R, V) : make_span<C, false>(R, V);
  for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
    const uint4 a = lds128(R.sc + j * 16);
    const uint4 b = X.cfg ? lds128(R.su + j * 16) : a;
    const int v0 = j * C::W - S.head;
#pragma unroll
    for (int i = 0; i < C::W; ++i) f(v0 + i, z2_of(X, velem<C>(a, i), X.cfg ? velem<C>(b, i) : 0.f));
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    f(v, z2_smem<C>(X, R, v));
  }
}

// ---------------------------------------------------------------- reductions

template <class C>
__device__ __forceinline__ float2 red_max2(float a, float c, Smem<C>& sm, int& slot) {
  a = warp_max(a);
  c = warp_max(c);
  float* s = sm.red8 + slot * 8 * C::NW;
  slot ^= 1;
  if ((threadIdx.x & 31) == 0) {
    s[gtid<C>() >> 5] = a;
    s[C::NW + (gtid<C>() >> 5)] = c;
  }
  csync<C>();
  float ra = s[0], rc = s[C::NW];
#pragma unroll
  for (int q = 1; q < C::NW; ++q) {
    ra = fmaxf(ra, s[q]);
    rc = fmaxf(rc, s[C::NW + q]);
  }
  return make_float2(ra, rc);
}

template <class C>
__device__ __forceinline__ float red_max1(float v, Smem<C>& sm, int& slot) {
  return red_max2<C>(v, kNegInf, sm, slot).x;
}

template <class C>
__device__ __forceinline__ unsigned long long red_max_u64(unsigned long long v, Smem<C>& sm, int& slot) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, v, o);
    v = x > v ? x : v;
  }
  unsigned long long* s = sm.redu + slot * C::NW;
  slot ^= 1;
  if ((threadIdx.x & 31) == 0) s[gtid<C>() >> 5] = v;
  csync<C>();
  unsigned long long r = s[0];
#pragma unroll
  for (int q = 1; q < C::NW; ++q) r = s[q] > r ? s[q] : r;
  return r;
}

// Sum of 8 floats over the block (one barrier).
template <class C>
__device__ __forceinline__ void block_sum8(float (&v)[8], Smem<C>& sm, int& slot) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = warp_sum(v[j]);
  float* s = sm.red8 + slot * 8 * C::NW;
  slot ^= 1;
  const int w = gtid<C>() >> 5;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j * C::NW + w] = v[j];
  }
  csync<C>();
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    float a = 0.f;
#pragma unroll
    for (int q = 0; q < C::NW; ++q) a += s[j * C::NW + q];
    v[j] = a;
  }
}

template <class C>
__device__ __forceinline__ float block_sum1(float v, Smem<C>& sm, int& slot) {
  float a[8] = {v, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  block_sum8<C>(a, sm, slot);
  return a[0];
}

// Group merge of per-thread (reference, sum) pairs: sum_t s_t * 2^(ref_t - M*scale)
// with M the group maximum of the per-thread maxima m_t.  Threads whose
// maximum is -inf hold s_t = 0 (or NaN) and are added unscaled.  Each warp
// rescales to its own maximum first; one barrier; the warp records are then
// merged the same way (the rounded products m*scale cancel level to level).
// Also clears the group's band counter (sm.misc[0]).
struct Stats3 {
  float m[3];    // per-thread maxima (cond, uncond, z2) -> group maxima
  float ref[3];  // per-thread references, m*scale rounded (0 when m is not finite)
  float s[3];    // per-thread sums relative to ref -> group sums relative to the maxima
};

template <class C>
__device__ __forceinline__ void group_merge3(Stats3& t, const float (&mscale)[3], Smem<C>& sm, int& slot) {
  const float kPosInf = __int_as_float(0x7f800000);
  const int w = gtid<C>() >> 5, lane = threadIdx.x & 31;
  float* b = sm.red8 + slot * 8 * C::NW;
  slot ^= 1;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float Mw = warp_max(t.m[j]);
    float s = t.s[j];
    if (t.m[j] > kNegInf && Mw < kPosInf) s = __fmul_rn(s, ex2_approx(__fsub_rn(t.ref[j], __fmul_rn(Mw, mscale[j]))));
    s = warp_sum(s);
    if (lane == 0) {
      b[j * C::NW + w] = Mw;
      b[(3 + j) * C::NW + w] = s;
    }
  }
  csync<C>();
  // every read of the previous position's band counter precedes this barrier,
  // and the next band pass follows a later one
  if (gtid<C>() == 0) sm.misc[0] = 0;
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float mq = lane < C::NW ? b[j * C::NW + lane] : kNegInf;
    const float sq = lane < C::NW ? b[(3 + j) * C::NW + lane] : 0.f;
    float M = mq;
#pragma unroll
    for (int o = 1; o < C::NW; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    float f = sq;
    if (mq > kNegInf && M < kPosInf)
      f = __fmul_rn(sq, ex2_approx(__fsub_rn(__fmul_rn(mq, mscale[j]), __fmul_rn(M, mscale[j]))));
#pragma unroll
    for (int o = 1; o < C::NW; o <<= 1) f += __shfl_xor_sync(0xffffffffu, f, o);
    t.m[j] = __shfl_sync(0xffffffffu, M, 0);
    t.s[j] = __shfl_sync(0xffffffffu, f, 0);
  }
}

// ---------------------------------------------------------------- scoring

struct Pick {
  float score;
  float vals;  // order key for exact score ties (sorted-candidate rule)
  int v;
};
__device__ __forceinline__ bool pick_better(const Pick& a, const Pick& b, bool turbo) {
  if (a.score > b.score) return true;
  if (a.score < b.score) return false;
  if (turbo && a.vals != b.vals) return a.vals > b.vals;
  return a.v < b.v;
}

__device__ __noinline__ float philox_noise_nl(uint64_t seed, uint64_t offset, int pos, int v) {
  return philox_token_gumbel(seed, offset, (uint32_t)pos, (uint32_t)v);
}

// Token noise; INL inlines the Philox rounds (hot callers whose live
// registers a call would spill), otherwise one out-of-line copy is shared.
template <bool INL = false>
__device__ __forceinline__ float noise_at(const SampleParams& P, int b, int pos, int l, int v) {
  if (P.noise_kind == YAPD_NOISE_EXPLICIT)
    return __ldg(P.gumbel_tok + (int64_t)b * P.gt_stride_req + (int64_t)l * P.gt_stride_pos + v);
  if (INL) return philox_token_gumbel(P.seed, P.offset, (uint32_t)pos, (uint32_t)v);
  return philox_noise_nl(P.seed, P.offset, pos, v);
}

// Whether token v is in request b's history (bitmap word or byte, from global memory).
__device__ __forceinline__ bool hist_bit(const SampleParams& P, int b, int v) {
  if (P.history_kind == YAPD_HISTORY_BITMAP) {
    const uint32_t* h = reinterpret_cast<const uint32_t*>(P.history) + (int64_t)b * P.history_stride;
    return (__ldg(h + (v >> 5)) >> (v & 31)) & 1u;
  }
  const uint8_t* h = reinterpret_cast<const uint8_t*>(P.history) + (int64_t)b * P.history_stride;
  return __ldg(h + v) != 0;
}

struct ScoreCtx {
  int b, pos, l;
  bool pen_on, noisy, turbo, minp_on;
  float rep, rrep;
  float r, minp_thr;  // min-p: keep iff 2^(z2-zmax) * r >= minp_thr
  const uint32_t* hbits;  // the request's history bitmap in shared memory, or null (global)
};

// Whether token v is in the request's history, from the shared-memory copy
// of its bitmap when the caller staged one.
__device__ __forceinline__ bool hist_bit_k(const SampleParams& P, const ScoreCtx& K, int v) {
  return K.hbits ? ((K.hbits[v >> 5] >> (v & 31)) & 1u) != 0u : hist_bit(P, K.b, v);
}

// The memory-borne inputs of a token's score (history bit, noise), fetched
// ahead of the arithmetic so that their latency overlaps other work.
struct ScoreIn {
  bool hb;
  float nz;
};
template <bool INL = false>
__device__ __forceinline__ ScoreIn score_in(const SampleParams& P, const ScoreCtx& K, int v) {
  ScoreIn r;
  r.hb = K.pen_on ? hist_bit_k(P, K, v) : false;
  r.nz = K.noisy ? noise_at<INL>(P, K.b, K.pos, K.l, v) : 0.f;
  return r;
}
__device__ __forceinline__ float score_from(const ScoreCtx& K, float vals, const ScoreIn& in) {
  float s = vals;
  if (K.pen_on && in.hb) s = penalize(vals, K.rep, K.rrep);
  if (K.noisy) s = __fadd_rn(s, in.nz);
  return s;
}

template <class C, bool INL = false>
__device__ __forceinline__ float exact_score(const SampleParams& P, const ScoreCtx& K, int v, float vals) {
  return score_from(K, vals, score_in<INL>(P, K, v));
}

template <class C>
__device__ __forceinline__ float approx_score(const SampleParams& P, const PosCtx& X, const ScoreCtx& K, int v,
                                              float z) {
  float va = __fmaf_rn(z, kLn2, X.Kval);
  if (K.pen_on && hist_bit_k(P, K, v)) va = va > 0.f ? __fmul_rn(va, K.rrep) : __fmul_rn(va, K.rep);
  return K.noisy ? __fadd_rn(va, noise_at(P, K.b, K.pos, K.l, v)) : va;
}

__device__ __forceinline__ float score_margin(float s) { return 2e-3f + 4e-5f * fabsf(s); }

// Block argmax of per-thread Picks; -1 when nothing was picked.
template <class C>
__device__ __forceinline__ int block_pick(const Pick& bp, bool turbo, Smem<C>& sm, int& slot) {
  const bool has = bp.score > kNegInf && bp.score == bp.score;
  const uint32_t ks = has ? ord_key(bp.score) : 0u;
  const uint32_t kv = has && turbo ? ord_key(bp.vals) : 0u;
  const unsigned long long me = ((unsigned long long)ks << 32) | kv;
  const unsigned long long w1 = red_max_u64<C>(has ? me : 0ull, sm, slot);
  if (w1 == 0ull) return -1;
  const unsigned long long w2 =
      red_max_u64<C>((has && me == w1) ? (unsigned long long)(uint32_t)(0x7fffffff - bp.v) : 0ull, sm, slot);
  return 0x7fffffff - (int)(uint32_t)w2;
}

// History bits of tokens v4 .. v4+3 (bit i: token v4 + i).
__device__ __forceinline__ unsigned hist4(const SampleParams& P, int b, int v4) {
  if (P.history_kind == YAPD_HISTORY_BITMAP) {
    const uint32_t* h = reinterpret_cast<const uint32_t*>(P.history) + (int64_t)b * P.history_stride;
    return (__ldg(h + (v4 >> 5)) >> (v4 & 31)) & 15u;
  }
  const uint8_t* h = reinterpret_cast<const uint8_t*>(P.history) + (int64_t)b * P.history_stride;
  unsigned m = 0u;
#pragma unroll
  for (int i = 0; i < 4; ++i) m |= (v4 + i < P.V && __ldg(h + v4 + i) != 0) ? (1u << i) : 0u;
  return m;
}

// The Gumbel noise of the tokens v4 + i with bit i of `keep` set (v4 a
// multiple of 4): one Philox block, the logarithms only for those tokens
// (one at a time, so a warp pays for the most any lane keeps, not for four).
__device__ __forceinline__ void noise4_kept(const SampleParams& P, const ScoreCtx& K, int v4, unsigned keep,
                                            float (&g)[4]) {
  if (P.noise_kind == YAPD_NOISE_EXPLICIT) {
    const float* row = P.gumbel_tok + (int64_t)K.b * P.gt_stride_req + (int64_t)K.l * P.gt_stride_pos;
#pragma unroll
    for (int i = 0; i < 4; ++i) g[i] = ((keep >> i) & 1u) ? __ldg(row + v4 + i) : 0.f;
    return;
  }
  const Philox4 r = philox4x32_10((uint32_t)v4 >> 2, (uint32_t)K.pos, (uint32_t)P.offset,
                                  (uint32_t)(P.offset >> 32) & 0x7fffffffu, (uint32_t)P.seed,
                                  (uint32_t)(P.seed >> 32));
  g[0] = g[1] = g[2] = g[3] = 0.f;
  while (keep) {
    const int i = __ffs(keep) - 1;
    keep &= keep - 1u;
    const uint32_t w = i == 0 ? r.x : i == 1 ? r.y : i == 2 ? r.z : r.w;
    const float gi = gumbel_from_uniform(uniform_from_word(w));
    g[0] = i == 0 ? gi : g[0];
    g[1] = i == 1 ? gi : g[1];
    g[2] = i == 2 ? gi : g[2];
    g[3] = i == 3 ? gi : g[3];
  }
}

// Cold argmax from the staged rows: elements with z2 >= H are kept (min-p
// test included); elements with band_lo <= z2 < H are kept iff their
// composite (exact value, -id) key is >= Xcomp.  Pass 1 runs over groups of
// four tokens per thread (one Philox block and one history word each) with
// approximate values and exact noise, keeping the tokens within a margin of
// the thread's best; pass 2 rescores those exactly (or every token, when a
// thread's list overflowed) and scans the boundary band.
template <class C>
__device__ __noinline__ int argmax_smem(const SampleParams& P, const PosCtx X, const RowRef<C> R, float H,
                                        float band_lo, unsigned long long Xcomp, const ScoreCtx& K, Pick bp, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  // nothing outside the band can be kept: the band's pick stands
  if (H >= kBig && !(band_lo < H)) return block_pick<C>(bp, K.turbo, sm, slot);
  const int V = P.V;
  constexpr int NC = 4;
  float best = kNegInf;
  int cv[NC];
  float cs[NC];  // their approximate scores: a list entry the best has left behind is dropped
  int nc = 0;
  bool ovf = false;
  for (int v4 = 4 * gtid<C>(); v4 < V; v4 += 4 * C::NT) {
    // the four tokens' z2 and filters first: no noise for a group none of
    // whose tokens is kept
    float zz[4];
    unsigned keep = 0u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = v4 + i;
      zz[i] = v < V ? z2_smem<C>(X, R, v) : kNegInf;
      bool in = v < V && zz[i] >= H;
      if (in && K.minp_on) in = __fmul_rn(ex2_approx(__fsub_rn(zz[i], X.zmax)), K.r) >= K.minp_thr;
      keep |= in ? (1u << i) : 0u;
    }
    if (!keep) continue;
    const unsigned hb = K.pen_on ? hist4(P, K.b, v4) : 0u;
    float va[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      va[i] = __fmaf_rn(zz[i], kLn2, X.Kval);
      if ((hb >> i) & 1u) va[i] = va[i] > 0.f ? __fmul_rn(va[i], K.rrep) : __fmul_rn(va[i], K.rep);
    }
    float g[4] = {0.f, 0.f, 0.f, 0.f};
    if (K.noisy && P.noise_kind != YAPD_NOISE_EXPLICIT && best > kNegInf) {
      // The Gumbel noise obeys G = -ln(-ln u) <= -ln(1 - u) (as -ln u >=
      // 1 - u): a token whose bound va - ln(1 - u) stays below the thread's
      // threshold (the best so far less its margin, less the rounding of
      // va + G) cannot pass the test below, and skips the logarithms.
      const Philox4 r = philox4x32_10((uint32_t)v4 >> 2, (uint32_t)K.pos, (uint32_t)P.offset,
                                      (uint32_t)(P.offset >> 32) & 0x7fffffffu, (uint32_t)P.seed,
                                      (uint32_t)(P.seed >> 32));
      const float thr = best - score_margin(best);
      const float tiny = 1e-6f * fabsf(thr) + 1e-6f;
      unsigned todo = keep;
      while (todo) {
        const int i = __ffs(todo) - 1;
        todo &= todo - 1u;
        const uint32_t w = i == 0 ? r.x : i == 1 ? r.y : i == 2 ? r.z : r.w;
        const float uu = uniform_from_word(w);
        const float vi = i == 0 ? va[0] : i == 1 ? va[1] : i == 2 ? va[2] : va[3];
        const float t = thr - vi - tiny;
        if (t > 0.0f && __fsub_rn(1.0f, uu) > ex2_approx(-t * kLog2e) * 1.0001f) {
          keep &= ~(1u << i);
          continue;
        }
        const float gi = gumbel_from_uniform(uu);
        g[0] = i == 0 ? gi : g[0];
        g[1] = i == 1 ? gi : g[1];
        g[2] = i == 2 ? gi : g[2];
        g[3] = i == 3 ? gi : g[3];
      }
    } else if (K.noisy) {
      noise4_kept(P, K, v4, keep, g);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int v = v4 + i;
      if (!((keep >> i) & 1u)) continue;
      const float sc = K.noisy ? __fadd_rn(va[i], g[i]) : va[i];
      // (the bound x - margin(x) rises with x: a token within the final
      // margin was within the margin of the running best when it came)
      if (!(sc >= best - score_margin(best))) continue;
      if (sc > best) {
        // a new best: drop the entries below its margin (they cannot be
        // within the final margin either), keeping the list short
        best = sc;
        const float lo = best - score_margin(best);
        int m = 0;
#pragma unroll
        for (int q = 0; q < NC; ++q)
          if (q < nc && cs[q] >= lo) {
            cv[m] = cv[q];
            cs[m] = cs[q];
            ++m;
          }
        nc = m;
      }
      if (nc < NC) {
        cv[nc] = v;
        cs[nc] = sc;
        ++nc;
      } else {
        ovf = true;
      }
    }
  }
  const float gbest = red_max1<C>(best, sm, slot);
  const float thr = gbest > kNegInf ? gbest - score_margin(gbest) : kBig;
  const bool all = csync_or<C>(ovf);
  auto rescore = [&](int v, float z) {
    float vals;
    const bool in_main = z >= H;
    if (in_main) {
      if (!(approx_score<C>(P, X, K, v, z) >= thr)) return;
      vals = exact_val<C>(P, X, R, v);
    } else {
      vals = exact_val<C>(P, X, R, v);
      if (cand_key(vals, v) < Xcomp) return;
    }
    const float es = exact_score<C>(P, K, v, vals);
    const Pick cand{es, vals, v};
    if (es == es && es > kNegInf && pick_better(cand, bp, K.turbo)) bp = cand;
  };
  if (!all) {
    for (int q = 0; q < nc; ++q) rescore(cv[q], z2_smem<C>(X, R, cv[q]));
  }
  if (all || band_lo < H) {
    for_each_z<C>(X, R, V, [&](int v, float z) {
      const bool in_main = z >= H;
      const bool in_band = z >= band_lo && z < H;
      if (!(in_band || (all && in_main))) return;
      if (K.minp_on && !(__fmul_rn(ex2_approx(__fsub_rn(z, X.zmax)), K.r) >= K.minp_thr)) return;
      rescore(v, z);
    });
  }
  return block_pick<C>(bp, K.turbo, sm, slot);
}

// Best kept band element (exact; band sorted in sm.cand with flags in sm.cflag).
template <class C>
__device__ __forceinline__ Pick band_pick(const SampleParams& P, const ScoreCtx& K, int nband, Smem<C>& sm) {
  Pick bp{kNegInf, kNegInf, 0x7fffffff};
  for (int q = gtid<C>(); q < nband; q += C::NT) {
    if (!sm.cflag[q]) continue;
    const unsigned long long c = sm.cand[q];
    const int v = cand_id(c);
    const float vals = cand_val(c);
    const float s = exact_score<C>(P, K, v, vals);
    const Pick cand{s, vals, v};
    if (s == s && s > kNegInf && pick_better(cand, bp, K.turbo)) bp = cand;
  }
  return bp;
}

// ---------------------------------------------------------------- bands

struct Band {
  int n;          // elements in the band (<= BAND unless overflow)
  float H;        // z2 >= H: outside and above the band
  float n_above;  // count of z2 >= H
  float m_above;  // mass (2^(z2-zmax)) of z2 >= H
  bool overflow;
};

// Sort sm.cand[0..n) descending with sm.cande alongside (one thread per element).
template <class C>
__device__ __forceinline__ void rank_sort(int n, Smem<C>& sm) {
  const int tid = gtid<C>();
  unsigned long long key = 0ull;
  float ev = 0.f;
  int rank = 0;
  if (tid < n) {
    key = sm.cand[tid];
    ev = sm.cande[tid];
    for (int j = 0; j < n; ++j) rank += (sm.cand[j] > key) ? 1 : 0;
  }
  csync<C>();
  if (tid < n) {
    sm.cand[rank] = key;
    sm.cande[rank] = ev;
  }
  csync<C>();
}

// Cold band from the staged rows: {lo_z <= z2 < hi_z}, with count and mass above hi_z.
template <class C>
__device__ __noinline__ Band band_smem(const SampleParams& P, const PosCtx X, const RowRef<C> R, float lo_z,
                                       float hi_z, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  const int V = P.V;
  csync<C>();
  if (gtid<C>() == 0) sm.misc[0] = 0;
  csync<C>();
  float na = 0.f, ma = 0.f;
  for_each_z<C>(X, R, V, [&](int v, float z) {
    if (z >= hi_z) {
      na += 1.f;
      ma += ex2_approx(__fsub_rn(z, X.zmax));
    } else if (z >= lo_z) {
      const int at = atomicAdd(&sm.misc[0], 1);
      if (at < C::BAND) {
        sm.cand[at] = cand_key(exact_val<C>(P, X, R, v), v);
        sm.cande[at] = ex2_approx(__fsub_rn(z, X.zmax));
      }
    }
  });
  float acc[8] = {na, ma, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  block_sum8<C>(acc, sm, slot);
  Band bd;
  bd.n = sm.misc[0];
  bd.overflow = bd.n > C::BAND;
  if (bd.overflow) bd.n = C::BAND;
  bd.H = hi_z;
  bd.n_above = acc[0];
  bd.m_above = acc[1];
  if (!bd.overflow) rank_sort<C>(bd.n, sm);
  return bd;
}

// Per band element (sorted position q): kept by top-k (q < k_left), top-p
// (cum_before < top_p over the band's prefix on top of the mass above it)
// and min-p (p >= minp_thr).  Writes sm.cflag[q].
template <class C>
__device__ __forceinline__ void band_flags(const Band& bd, bool use_k, int k_left, bool topp_on, float top_p,
                                           float r, bool minp_on, float minp_thr, Smem<C>& sm) {
  const int tid = gtid<C>();
  if (tid < 32) {
    double run = (double)bd.m_above * (double)r;
    for (int q0 = 0; q0 < bd.n; q0 += 32) {
      const int q = q0 + tid;
      const float p = q < bd.n ? __fmul_rn(sm.cande[q], r) : 0.f;
      double incl = (double)p;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, incl, o);
        if (tid >= o) incl += n;
      }
      incl += run;
      if (q < bd.n) {
        bool keep = true;
        if (use_k) keep = keep && (q < k_left);
        if (topp_on) keep = keep && (__fsub_rn((float)incl, p) < top_p);
        if (minp_on) keep = keep && (p >= minp_thr);
        sm.cflag[q] = keep ? 1 : 0;
      }
      run = __shfl_sync(0xffffffffu, incl, 31);
    }
  }
  csync<C>();
}

// Counts and masses of {z2 >= t[j]} over the staged rows.
template <class C>
__device__ __forceinline__ void stats4_smem(const PosCtx& X, const RowRef<C>& R, int V, const float (&t)[4],
                                            float (&cnt)[4], float (&mass)[4], Smem<C>& sm, int& slot) {
  float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int v = gtid<C>(); v < V; v += C::NT) {
    const float z = z2_smem<C>(X, R, v);
    const float e = ex2_approx(__fsub_rn(z, X.zmax));
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const bool in = z >= t[j];
      a[j] += in ? 1.f : 0.f;
      a[4 + j] += in ? e : 0.f;
    }
  }
  block_sum8<C>(a, sm, slot);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    cnt[j] = a[j];
    mass[j] = a[4 + j];
  }
}

// Bracket the z2 where stat(z2 >= t) (count or mass) crosses the target:
// on return stat(hi) < tgt_lo and stat(lo) >= tgt_hi, with few elements
// between them unless the values are (near) ties.
template <class C>
__device__ __noinline__ void bracket_smem(const PosCtx X, const RowRef<C> R, int V, bool by_mass, float tgt_lo,
                                          float tgt_hi, float floor_t, float cnt_floor, float& lo, float& hi, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  lo = floor_t;
  float cnt_lo = cnt_floor;
  hi = X.zmax + 1.0f;
  float cnt_hi = 0.f;
  constexpr int kTarget = C::BAND / 2;
  for (int round = 0; round < 12; ++round) {
    float t[4];
    if (round == 0) {
      const float L[4] = {2.f, 6.f, 12.f, 24.f};
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = fmaxf(__fsub_rn(X.zmax, L[j]), floor_t);
    } else {
      const float lo_e = fmaxf(lo, __fsub_rn(hi, 64.f));
#pragma unroll
      for (int j = 0; j < 4; ++j) t[j] = lo_e + (hi - lo_e) * (float)(j + 1) * 0.2f;
    }
    float cnt[4], mass[4];
    stats4_smem<C>(X, R, V, t, cnt, mass, sm, slot);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float F = by_mass ? mass[j] : cnt[j];
      if (F >= tgt_hi && t[j] > lo) {
        lo = t[j];
        cnt_lo = cnt[j];
      }
      if (F < tgt_lo && t[j] < hi) {
        hi = t[j];
        cnt_hi = cnt[j];
      }
    }
    if (cnt_lo - cnt_hi <= (float)kTarget) break;
    if (hi - lo <= 8.f * zmargin(hi)) break;
  }
}

// Massive-tie fallback for a band too large for shared memory: composite
// (exact value, -id) thresholds by bisection (top-k by count, top-p by the
// exclusive prefix mass).  Band elements with composite >= the result are kept.
template <class C>
__device__ __noinline__ unsigned long long overflow_resolve(const SampleParams& P, const PosCtx X,
                                                            const RowRef<C> R, float lo_z, float hi_z,
                                                            float n_above, float m_above, bool topk_on, int kk,
                                                            bool topp_on, float top_p, float S_all, float& Sk_out, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  const int V = P.V;
  unsigned long long Xk = 0ull;
  float Sn = S_all;
  if (topk_on) {
    const int need = kk - (int)n_above;
    if (need <= 0) {
      Xk = ~0ull;
    } else {
      unsigned long long lo = 0ull, hi = ~0ull;
      while (lo < hi) {
        const unsigned long long mid = lo + (hi - lo) / 2ull + 1ull;
        float cnt = 0.f;
        for (int v = gtid<C>(); v < V; v += C::NT) {
          const float z = z2_smem<C>(X, R, v);
          if (z >= lo_z && z < hi_z) cnt += (cand_key(exact_val<C>(P, X, R, v), v) >= mid) ? 1.f : 0.f;
        }
        if (block_sum1<C>(cnt, sm, slot) >= (float)need) lo = mid;
        else hi = mid - 1ull;
      }
      Xk = lo;
    }
    float m = 0.f;
    for (int v = gtid<C>(); v < V; v += C::NT) {
      const float z = z2_smem<C>(X, R, v);
      if (z >= lo_z && z < hi_z && cand_key(exact_val<C>(P, X, R, v), v) >= Xk)
        m += ex2_approx(__fsub_rn(z, X.zmax));
    }
    Sn = __fadd_rn(m_above, block_sum1<C>(m, sm, slot));
  }
  Sk_out = Sn;
  unsigned long long Xr = Xk;
  if (topp_on) {
    const double tgt = (double)top_p * (double)Sn;
    unsigned long long lo = 0ull, hi = ~0ull;
    while (lo < hi) {
      const unsigned long long mid = lo + (hi - lo) / 2ull;
      float m = 0.f;
      for (int v = gtid<C>(); v < V; v += C::NT) {
        const float z = z2_smem<C>(X, R, v);
        if (z >= lo_z && z < hi_z) {
          const unsigned long long ck = cand_key(exact_val<C>(P, X, R, v), v);
          if (ck > mid && ck >= Xk) m += ex2_approx(__fsub_rn(z, X.zmax));
        }
      }
      if ((double)m_above + (double)block_sum1<C>(m, sm, slot) < tgt) hi = mid;
      else lo = mid + 1ull;
    }
    Xr = lo > Xr ? lo : Xr;
  }
  return Xr;
}

// Lowest id whose z2 is NaN, else +inf, else -1 (torch orders NaN first).
template <class C>
__device__ __noinline__ int first_nan_or_inf(const PosCtx X, const RowRef<C> R, int V, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  int fn = 0x7fffffff, fi = 0x7fffffff;
  for (int v = gtid<C>(); v < V; v += C::NT) {
    const float z = z2_smem<C>(X, R, v);
    if (!(z == z) && v < fn) fn = v;
    if (z == __int_as_float(0x7f800000) && v < fi) fi = v;
  }
  const unsigned long long w = red_max_u64<C>(
      ((unsigned long long)(uint32_t)(0x7fffffff - fn) << 32) | (uint32_t)(0x7fffffff - fi), sm, slot);
  const int n = 0x7fffffff - (int)(uint32_t)(w >> 32);
  if (n != 0x7fffffff) return n;
  // no NaN anywhere: the largest +inf record wins the low half only if no thread saw NaN
  const unsigned long long w2 = red_max_u64<C>((unsigned long long)(uint32_t)(0x7fffffff - fi), sm, slot);
  const int i = 0x7fffffff - (int)(uint32_t)w2;
  return i == 0x7fffffff ? -1 : i;
}

// First sorted candidate (largest exact value, lowest id): torch's argmax over
// an all -inf row returns it.
template <class C>
__device__ __noinline__ int top1_smem(const SampleParams& P, const PosCtx X, const RowRef<C> R, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  unsigned long long best = 0ull;
  const float zlo = __fsub_rn(X.zmax, zmargin(X.zmax));
  for (int v = gtid<C>(); v < P.V; v += C::NT) {
    const float z = z2_smem<C>(X, R, v);
    if (z >= zlo) {
      const unsigned long long k = cand_key(exact_val<C>(P, X, R, v), v);
      best = k > best ? k : best;
    }
  }
  const unsigned long long w = red_max_u64<C>(best, sm, slot);
  const int id = cand_id(w);
  return (w == 0ull || id < 0 || id >= P.V) ? 0 : id;
}

// Top-k / top-p (and min-p) selection from the staged rows.
// Histogram bracket: the same contract as bracket_smem (lo, hi around the
// point where the count (or mass) of {z2 >= t} crosses the target), from
// passes that bin z2 into kHistBins equal bins below zmax + 1 (counts and
// masses by shared-memory atomics) and refine inside the crossing bins; false
// when the target lies below the binned range (the caller then probes).
template <class C>
__device__ __noinline__ bool bracket_hist(const PosCtx X, const RowRef<C> R, int V, bool by_mass, float tgt_lo,
                                          float tgt_hi, float floor_t, float& lo, float& hi, Smem<C>& sm) {
  constexpr int NB = kHistBins, PER = NB / 32;
  constexpr int kTarget = C::BAND / 2;
  const int tid = gtid<C>(), lane = threadIdx.x & 31;
  float top = __fadd_rn(X.zmax, 1.0f);
  float base = fmaxf(floor_t, __fsub_rn(X.zmax, 63.0f));
  float above_c = 0.f, above_m = 0.f;  // count / mass of {z2 >= top}
  bool ok = false;
  for (int pass = 0; pass < 3; ++pass) {
    if (!(top > base)) break;
    const float w = __fdiv_rn(__fsub_rn(top, base), (float)NB);
    const float iw = __fdiv_rn(1.0f, w);
    for (int i = tid; i < NB; i += C::NT) {
      sm.hc[i] = 0;
      sm.hm[i] = 0.f;
    }
    csync<C>();
    for_each_z<C>(X, R, V, [&](int, float z) {
      if (z >= base && z < top) {
        const int bi = min(max((int)__fmul_rn(__fsub_rn(z, base), iw), 0), NB - 1);
        atomicAdd(&sm.hc[bi], 1);
        if (by_mass) atomicAdd(&sm.hm[bi], ex2_approx(__fsub_rn(z, X.zmax)));
      }
    });
    csync<C>();
    // lane s of the group's first warp scans bins NB-1-s*PER downwards; the
    // running totals G(j) = F(base + j*w) grow towards lower bins
    if (tid < 32) {
      float segc = 0.f, segm = 0.f;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int bi = NB - 1 - (lane * PER + k);
        segc += (float)sm.hc[bi];
        segm += sm.hm[bi];
      }
      float pc = segc, pm = segm;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float yc = __shfl_up_sync(0xffffffffu, pc, o);
        const float ym = __shfl_up_sync(0xffffffffu, pm, o);
        if (lane >= o) {
          pc += yc;
          pm += ym;
        }
      }
      float gc = above_c + pc - segc, gm = above_m + pm - segm;  // G at the top of this segment
      int jlo = -1, jx = -1;
      float gclo = 0.f, gcx = 0.f, gmx = 0.f;
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int bi = NB - 1 - (lane * PER + k);
        const float gc0 = gc, gm0 = gm;  // G(bi + 1)
        gc += (float)sm.hc[bi];
        gm += sm.hm[bi];
        const float F = by_mass ? gm : gc;
        if (jx < 0 && F >= tgt_lo) {
          jx = bi;
          gcx = gc0;
          gmx = gm0;
        }
        if (jlo < 0 && F >= tgt_hi) {
          jlo = bi;
          gclo = gc;
        }
      }
      // the first lane (highest bins) holding each crossing
      const unsigned blo = __ballot_sync(0xffffffffu, jlo >= 0), bx = __ballot_sync(0xffffffffu, jx >= 0);
      if (lane == 0) sm.misc[4] = blo ? 1 : 0;
      if (blo) {
        const int sl = __ffs(blo) - 1, sx = __ffs(bx) - 1;
        const int jl = __shfl_sync(0xffffffffu, jlo, sl);
        const float cl = __shfl_sync(0xffffffffu, gclo, sl);
        const int jh = __shfl_sync(0xffffffffu, jx, sx) + 1;
        const float ch = __shfl_sync(0xffffffffu, gcx, sx), mh = __shfl_sync(0xffffffffu, gmx, sx);
        if (lane == 0) {
          sm.red8[0] = __fadd_rn(base, __fmul_rn((float)jl, w));
          sm.red8[1] = jh >= NB ? top : __fadd_rn(base, __fmul_rn((float)jh, w));
          sm.red8[2] = __fsub_rn(cl, ch);
          sm.red8[3] = ch;
          sm.red8[4] = mh;
        }
      }
    }
    csync<C>();
    if (!sm.misc[4]) break;  // the target lies below the binned range
    ok = true;
    lo = sm.red8[0];
    hi = sm.red8[1];
    const float between = sm.red8[2];
    above_c = sm.red8[3];
    above_m = sm.red8[4];
    csync<C>();  // every read of the record precedes the next pass's writes
    if (between <= (float)kTarget || hi - lo <= 8.f * zmargin(hi)) break;
    base = lo;
    top = hi;
  }
  return ok;
}

template <class C>
__device__ __noinline__ int select_cold(const SampleParams& P, const PosCtx X, const RowRef<C> R, ScoreCtx K,
                                        int topk_raw, bool topk_on, bool topp_on, float top_p, float min_p, Smem<C>& sm) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  const int V = P.V;
  float H = -kBig, band_lo = kBig;
  unsigned long long Xcomp = 0ull;
  int nband = 0;
  float Sn = X.S;
  K.r = __fdiv_rn(1.0f, Sn);
  float Hk = -kBig, cnt_k = (float)V;
  Band bk{};
  int k_left = 0;
  bool done = false;
  if (topk_on) {
    float lo, hi;
    if (!bracket_hist<C>(X, R, V, false, (float)topk_raw, (float)topk_raw, -kBig, lo, hi, sm))
      bracket_smem<C>(X, R, V, false, (float)topk_raw, (float)topk_raw, -kBig, (float)V, lo, hi, sm);
    csync<C>();
    const float blo = __fsub_rn(lo, zmargin(lo)), bhi = __fadd_rn(hi, zmargin(hi));
    // a small k: the whole top-k set (everything from the boundary band up)
    // in the sorted list when it fits, so that top-k, top-p and min-p are
    // all decided on it and no pass over the row is left for the sample
    const bool whole = topk_raw <= C::BAND - 16;
    bk = band_smem<C>(P, X, R, blo, whole ? kBig : bhi, sm);
    csync<C>();
    if (whole && bk.overflow) {
      bk = band_smem<C>(P, X, R, blo, bhi, sm);
      csync<C>();
    }
    if (bk.overflow) {
      float Sk;
      Xcomp = overflow_resolve<C>(P, X, R, blo, bhi, bk.n_above, bk.m_above, true, topk_raw,
                                  topp_on && bk.m_above < __fmul_rn(top_p, X.S), top_p, X.S, Sk, sm);
      csync<C>();
      Sn = Sk;
      K.r = __fdiv_rn(1.0f, Sn);
      if (K.minp_on) K.minp_thr = __fmul_rn(min_p, K.r);
      H = bhi;
      band_lo = blo;
      nband = 0;
      done = true;
    } else {
      k_left = topk_raw - (int)bk.n_above;
      float part = 0.f;
      for (int q = gtid<C>(); q < bk.n && q < k_left; q += C::NT) part += sm.cande[q];
      Sn = __fadd_rn(bk.m_above, block_sum1<C>(part, sm, slot));
      K.r = __fdiv_rn(1.0f, Sn);
      Hk = bk.H;
      cnt_k = bk.n_above;
    }
  }
  if (!done) {
    const float p0 = (topk_on && bk.n_above == 0.f && bk.n > 0) ? __fmul_rn(sm.cande[0], K.r) : K.r;
    if (K.minp_on) K.minp_thr = __fmul_rn(min_p, p0);
    const float tgt = __fmul_rn(top_p, Sn);
    if (topp_on && !(topk_on && bk.m_above < __fmul_rn(tgt, 1.00001f))) {
      float lo, hi;
      if (!bracket_hist<C>(X, R, V, true, __fmul_rn(tgt, 0.99999f), __fmul_rn(tgt, 1.00001f), Hk, lo, hi, sm))
        bracket_smem<C>(X, R, V, true, __fmul_rn(tgt, 0.99999f), __fmul_rn(tgt, 1.00001f), Hk, cnt_k, lo, hi, sm);
    csync<C>();
      const float blo = fmaxf(__fsub_rn(lo, zmargin(lo)), Hk), bhi = __fadd_rn(hi, zmargin(hi));
      const Band bp = band_smem<C>(P, X, R, blo, bhi, sm);
    csync<C>();
      if (bp.overflow) {
        float Sk;
        Xcomp = overflow_resolve<C>(P, X, R, blo, bhi, bp.n_above, bp.m_above, false, 0, true, top_p, Sn, Sk, sm);
      csync<C>();
        H = bhi;
        band_lo = blo;
        nband = 0;
      } else {
        band_flags<C>(bp, false, 0, true, top_p, K.r, K.minp_on, K.minp_thr, sm);
        H = bp.H;
        nband = bp.n;
      }
    } else if (topk_on) {
      band_flags<C>(bk, true, k_left, topp_on, top_p, K.r, K.minp_on, K.minp_thr, sm);
      H = bk.H;
      nband = bk.n;
    } else {
      // min-p set too large for one band: min-p as an elementwise condition
      H = -kBig;
      nband = 0;
    }
  }
  const Pick bp0 = band_pick<C>(P, K, nband, sm);
  const int c = argmax_smem<C>(P, X, R, H, band_lo, Xcomp, K, bp0, sm);
  csync<C>();
  return c >= 0 ? c : top1_smem<C>(P, X, R, sm);
}

// Per-group scratch: reduction slots (0/1: hot path, 2/3: out-of-line paths),
// the band counter and the candidate band.
template <class C>
struct Smem {
  float red8[4 * 8 * C::NW];
  unsigned long long redu[4 * C::NW];
  int misc[8];
  unsigned long long cand[C::BAND];
  float cande[C::BAND];
  float2 cpc[32];             // PMI inputs of the first 32 band members
  float cscore[32];           // their exact scores (penalty + noise)
  unsigned char cflag[C::BAND];
  alignas(16) int hc[kHistBins];    // bracket histogram: counts ...
  union {
    alignas(16) float hm[kHistBins];     // ... and masses 2^(z2 - zmax) per bin (select_cold)
    alignas(16) uint32_t hq[kHistBins];  // ... or fixed-point masses (histogram select)
  };
  int hsi[8];                 // histogram select: the scan's crossings ...
  float hsf[8];               // ... and its mass bounds
  int klist[C::NT];           // histogram select: ids of the tokens above band P (kept)
  uint32_t kq[C::NW * kKqPerWarp];  // kept_pass: each warp's queue of (Philox block, keep mask) units
};

template <class C>
struct KSmem {
  uint64_t full[C::NSTAGE];   // rows landed (one expect_tx arrive + the copy bytes)
  uint64_t ready[C::NSTAGE];  // the group is done with the position (one arrive per group warp)
  Hand hand[C::NSTAGE];       // the group -> tail warp record of the stage's position
  int issued[C::NSTAGE];      // copies armed on full[s] ...
  int landed[C::NSTAGE];      // ... and waited for (read only after the final barrier)
  int nodyn;                  // claimed schedule: this CTA stopped claiming (other CTAs' entries were late)
  int own[C::NSTAGE];         // claimed schedule: this CTA's own first positions
  int scan[32];               // per-warp counts of the fused preamble
  Smem<C> g[C::NG];
  alignas(128) unsigned char stage[C::NSTAGE][C::STAGE_BYTES];
};

// softmax(c)[v], softmax(u)[v] as the reference rounds them (server/engine.py:539-540, 553, 556),
// from the token's cond / uncond logits.
template <bool CFG>
__device__ __forceinline__ float2 pmi_cu(const PosCtx& X, float cv, float uv) {
  const float pc = __fmul_rn(expf(__fsub_rn(cv, X.mc)), __fdiv_rn(1.0f, X.Sc));
  float pu = 0.f;
  if (CFG) pu = __fmul_rn(expf(__fsub_rn(uv, X.mu)), __fdiv_rn(1.0f, X.Su));
  return make_float2(pc, pu);
}

template <class C, bool CFG>
__device__ __forceinline__ float2 pmi_inputs(const PosCtx& X, const RowRef<C>& R, int v) {
  const float cv = load_elem_smem<C>(R.sc, R.gc, v);
  const float uv = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
  return pmi_cu<CFG>(X, cv, uv);
}

// Write the sampled id and the PMI inputs softmax(c)[s], softmax(u)[s]
// (server/engine.py:539-540, 553, 556); the unmask kernel forms the PMI.
template <class C, bool CFG>
__device__ __forceinline__ void write_choice(const SampleParams& P, const RowRef<C>& R, int pos, int chosen,
                                             float mc, float Sc, float mu, float Su) {
  P.sampled[pos] = chosen;
  if (P.pcu) {
    PosCtx X;
    X.mc = mc;
    X.Sc = Sc;
    X.mu = mu;
    X.Su = Su;
    P.pcu[pos] = pmi_inputs<C, CFG>(X, R, chosen);
  }
}

template <class C, bool CFG>
__device__ __forceinline__ RowRef<C> row_ref(const SampleParams& P, KSmem<C>& ks, int stage, int pos) {
  (void)P;
  (void)pos;
  RowRef<C> R;
  R.sc = ks.stage[stage];
  R.su = ks.stage[stage] + C::ROW_SLOT;
  R.gc = ks.hand[stage].gc;
  R.gu = CFG ? ks.hand[stage].gu : R.gc;
  return R;
}

template <class C, bool CFG>
__device__ __forceinline__ Span make_span(const RowRef<C>& R, int V) {
  Span S;
  if (CFG && R.gu.head != R.gc.head) {
    S.j0 = S.j1 = 0;
    S.head = 0;
    S.nlo = 0;
    S.hi0 = 0;
    S.nscal = V;
    return S;
  }
  const int head = R.gc.head;
  const int avail = CFG ? min(R.gc.avail, R.gu.avail) : R.gc.avail;
  S.head = head;
  S.j0 = head > 0 ? 1 : 0;
  S.nlo = min(S.j0 * C::W - head, V);
  int j1 = (avail + head) / C::W;
  if (j1 < S.j0) j1 = S.j0;
  S.j1 = j1;
  S.hi0 = max(j1 * C::W - head, S.nlo);
  S.nscal = S.nlo + (V - S.hi0);
  return S;
}

// Pass 1 of the two-pass form: this thread's maxima of c and u and minimum
// of u (NaN ignored).
template <class C, bool CFG>
__device__ __forceinline__ void pass_max(const RowRef<C>& R, const Span& S, float& mc, float& mu, float& nu) {
  const int tid = gtid<C>();
  if constexpr (C::BF16) {
    uint32_t c2 = 0xff80ff80u, u2 = 0xff80ff80u, n2 = 0x7f807f80u;
#pragma unroll 4
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      c2 = bmax2(c2, bmax2(bmax2(a.x, a.y), bmax2(a.z, a.w)));
      if (CFG) {
        const uint4 q = lds128(R.su + j * 16);
        u2 = bmax2(u2, bmax2(bmax2(q.x, q.y), bmax2(q.z, q.w)));
        n2 = bmin2(n2, bmin2(bmin2(q.x, q.y), bmin2(q.z, q.w)));
      }
    }
    mc = fmaxf(bf16lo(c2), bf16hi(c2));
    mu = fmaxf(bf16lo(u2), bf16hi(u2));
    nu = fminf(bf16lo(n2), bf16hi(n2));
  } else {
    float c0 = kNegInf, u0 = kNegInf, n0 = __int_as_float(0x7f800000);
#pragma unroll 4
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      c0 = fmax3(c0, __uint_as_float(a.x), __uint_as_float(a.y));
      c0 = fmax3(c0, __uint_as_float(a.z), __uint_as_float(a.w));
      if (CFG) {
        const uint4 q = lds128(R.su + j * 16);
        u0 = fmax3(u0, __uint_as_float(q.x), __uint_as_float(q.y));
        u0 = fmax3(u0, __uint_as_float(q.z), __uint_as_float(q.w));
        n0 = fmin3(n0, __uint_as_float(q.x), __uint_as_float(q.y));
        n0 = fmin3(n0, __uint_as_float(q.z), __uint_as_float(q.w));
      }
    }
    mc = c0;
    mu = u0;
    nu = n0;
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    mc = fmaxf(mc, load_elem_smem<C>(R.sc, R.gc, v));
    if (CFG) {
      const float u = load_elem_smem<C>(R.su, R.gu, v);
      mu = fmaxf(mu, u);
      nu = fminf(nu, u);
    }
  }
  if (!CFG) {
    mu = kNegInf;
    nu = 0.f;
  }
}

// Exact maximum of z2' = A2*c - B2*u over this thread's elements (NaN
// ignored); the reference point when the bound from pass 1 is unusable.
template <class C, bool CFG>
__device__ __noinline__ float thread_zmax(const PosCtx X, const RowRef<C> R, const Span S) {
  const int tid = gtid<C>();
  float m = kNegInf;
  for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
    const uint4 a = lds128(R.sc + j * 16);
    uint4 q = a;
    if (CFG) q = lds128(R.su + j * 16);
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      const float c = velem<C>(a, i);
      m = fmaxf(m, CFG ? __fmaf_rn(c, X.A2, __fmul_rn(velem<C>(q, i), -X.B2)) : __fmul_rn(c, X.A2));
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    m = fmaxf(m, CFG ? __fmaf_rn(c, X.A2, __fmul_rn(load_elem_smem<C>(R.su, R.gu, v), -X.B2))
                     : __fmul_rn(c, X.A2));
  }
  return m;
}

// Pass 2 of the two-pass form: sc = sum 2^(c*log2e + nmcL), su likewise,
// s = sum 2^d and dmax = max d with d = A2*c - B2*u + nzr (NaN ignored in the
// maximum, kept in the sums); vz[k] = the largest d of this thread's k-th
// vector (-inf past the row).
template <class C, bool CFG>
__device__ __forceinline__ void pass_sums(const PosCtx& X, const RowRef<C>& R, const Span& S, float nmcL,
                                          float nmuL, float nzr, float& sc, float& su, float& s, float& dmax,
                                          float (&vz)[C::KV]) {
  const int tid = gtid<C>();
  const float A2 = X.A2, nB2 = -X.B2;
  float sc0 = 0.f, sc1 = 0.f, su0 = 0.f, su1 = 0.f, s0 = 0.f, s1 = 0.f, dm = kNegInf;
  if constexpr (C::BF16) {
    // packed pairs: element 2t in the low half, 2t+1 in the high half, so the
    // two accumulators of each sum see the same additions as the scalar form
    const unsigned long long L2p = f2_pack(kLog2e, kLog2e), A2p = f2_pack(A2, A2), nB2p = f2_pack(nB2, nB2);
    const unsigned long long nmcLp = f2_pack(nmcL, nmcL), nmuLp = f2_pack(nmuL, nmuL), nzrp = f2_pack(nzr, nzr);
    unsigned long long scp = f2_pack(0.f, 0.f), sup = scp, sp = scp;
#pragma unroll
    for (int k = 0; k < C::KV; ++k) {
      const int j = S.j0 + tid + k * C::NT;
      vz[k] = kNegInf;
      if (j < S.j1) {
        const uint4 a = lds128(R.sc + j * 16);
        uint4 q = a;
        if (CFG) q = lds128(R.su + j * 16);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
        float m = kNegInf;
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const unsigned long long cx = f2_bf16(aw[t]);
          unsigned long long dx;
          float lo, hi;
          if (CFG) {
            const unsigned long long ux = f2_bf16(qw[t]);
            dx = f2_fma(cx, A2p, f2_fma(ux, nB2p, nzrp));
            f2_unpack(f2_fma(ux, L2p, nmuLp), lo, hi);
            sup = f2_add(sup, f2_pack(ex2_approx(lo), ex2_approx(hi)));
          } else {
            dx = f2_fma(cx, A2p, nzrp);
          }
          f2_unpack(f2_fma(cx, L2p, nmcLp), lo, hi);
          scp = f2_add(scp, f2_pack(ex2_approx(lo), ex2_approx(hi)));
          f2_unpack(dx, lo, hi);
          sp = f2_add(sp, f2_pack(ex2_approx(lo), ex2_approx(hi)));
          m = fmax3(m, lo, hi);
        }
        vz[k] = m;
        dm = fmaxf(dm, m);
      }
    }
    f2_unpack(scp, sc0, sc1);
    f2_unpack(sup, su0, su1);
    f2_unpack(sp, s0, s1);
  } else {
#pragma unroll
    for (int k = 0; k < C::KV; ++k) {
      const int j = S.j0 + tid + k * C::NT;
      vz[k] = kNegInf;
      if (j < S.j1) {
        const uint4 a = lds128(R.sc + j * 16);
        uint4 q = a;
        if (CFG) q = lds128(R.su + j * 16);
        float d[C::W];
#pragma unroll
        for (int i = 0; i < C::W; ++i) {
          const float c = velem<C>(a, i);
          d[i] = CFG ? __fmaf_rn(c, A2, __fmaf_rn(velem<C>(q, i), nB2, nzr)) : __fmaf_rn(c, A2, nzr);
        }
#pragma unroll
        for (int i = 0; i < C::W; i += 2) {
          sc0 += ex2_approx(__fmaf_rn(velem<C>(a, i), kLog2e, nmcL));
          sc1 += ex2_approx(__fmaf_rn(velem<C>(a, i + 1), kLog2e, nmcL));
          if (CFG) {
            su0 += ex2_approx(__fmaf_rn(velem<C>(q, i), kLog2e, nmuL));
            su1 += ex2_approx(__fmaf_rn(velem<C>(q, i + 1), kLog2e, nmuL));
          }
          s0 += ex2_approx(d[i]);
          s1 += ex2_approx(d[i + 1]);
        }
        float m = fmaxf(d[0], d[1]);
#pragma unroll
        for (int i = 2; i + 1 < C::W; i += 2) m = fmax3(m, d[i], d[i + 1]);
        vz[k] = m;
        dm = fmaxf(dm, m);
      }
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    sc0 += ex2_approx(__fmaf_rn(c, kLog2e, nmcL));
    float dv;
    if (CFG) {
      const float u = load_elem_smem<C>(R.su, R.gu, v);
      su0 += ex2_approx(__fmaf_rn(u, kLog2e, nmuL));
      dv = __fmaf_rn(c, A2, __fmaf_rn(u, nB2, nzr));
    } else {
      dv = __fmaf_rn(c, A2, nzr);
    }
    dm = fmaxf(dm, dv);
    s0 += ex2_approx(dv);
  }
  sc = sc0 + sc1;
  su = su0 + su1;
  s = s0 + s1;
  dmax = dm;
}

// Sum of 2^(A2*c - B2*u + nzr) alone (after an underflowed pass 2).
template <class C, bool CFG>
__device__ __noinline__ float pass_resum(const PosCtx X, const RowRef<C> R, const Span S, float nzr) {
  const int tid = gtid<C>();
  float s = 0.f;
  for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
    const uint4 a = lds128(R.sc + j * 16);
    uint4 q = a;
    if (CFG) q = lds128(R.su + j * 16);
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      const float c = velem<C>(a, i);
      s += ex2_approx(CFG ? __fmaf_rn(c, X.A2, __fmaf_rn(velem<C>(q, i), -X.B2, nzr)) : __fmaf_rn(c, X.A2, nzr));
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    s += ex2_approx(CFG ? __fmaf_rn(c, X.A2, __fmaf_rn(load_elem_smem<C>(R.su, R.gu, v), -X.B2, nzr))
                        : __fmaf_rn(c, X.A2, nzr));
  }
  return s;
}

// Add token v to the band: its exact value and mass, and for the first 32
// members also its exact score (penalty + noise) and PMI inputs, so that the
// finishing warp needs neither the staged rows nor global memory.
template <class C, bool CFG>
__device__ __forceinline__ void band_add(const SampleParams& P, const PosCtx& X, const RowRef<C>& R,
                                         const ScoreCtx& K, int v, Smem<C>& sm) {
  const int at = atomicAdd(&sm.misc[0], 1);
  if (at < C::BAND) {
    const float vals = exact_val<C>(P, X, R, v);
    sm.cand[at] = cand_key(vals, v);
    sm.cande[at] = ex2_approx(__fsub_rn(z2_smem<C>(X, R, v), X.zmax));
    if (at < 32) {
      sm.cscore[at] = exact_score<C, true>(P, K, v, vals);
      sm.cpc[at] = pmi_inputs<C, CFG>(X, R, v);
    }
  }
}

// The min-p band {z2 >= lo_z} from the vectors pass 2 marked (and
// every scalar element), unsorted in sm.cand (exact value, id) and sm.cande
// (2^(z2 - zmax)); returns its size (may exceed BAND).  sm.misc[0] must be
// zero on entry.
template <class C, bool CFG>
__device__ __forceinline__ int band_marked(const SampleParams& P, const PosCtx& X, const RowRef<C>& R,
                                           const ScoreCtx& K, const Span& S, uint32_t marks, float lo_z,
                                           Smem<C>& sm) {
  const int tid = gtid<C>();
  while (marks) {
    const int k = __ffs(marks) - 1;
    marks &= marks - 1u;
    const int j = S.j0 + tid + k * C::NT;
    const uint4 a = lds128(R.sc + j * 16);
    uint4 q = a;
    if (CFG) q = lds128(R.su + j * 16);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      const float z = z2_of(X, velem<C>(a, i), CFG ? velem<C>(q, i) : 0.f);
      m |= (z >= lo_z ? 1u : 0u) << i;
    }
    const int v0 = j * C::W - S.head;
    while (m) {
      const int i = __ffs(m) - 1;
      m &= m - 1u;
      band_add<C, CFG>(P, X, R, K, v0 + i, sm);
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    if (z2_smem<C>(X, R, v) >= lo_z) band_add<C, CFG>(P, X, R, K, v, sm);
  }
  csync<C>();
  return sm.misc[0];
}

// One position, worked by the calling group.
// Parts of the position context that need no statistics.
template <bool CFG>
__device__ __forceinline__ void item_ctx(const SampleParams& P, const ItemParams& Q, PosCtx& X, float& sA) {
  X.cfg = CFG;
  X.T = Q.T;
  X.scale = X.T > 0.0f;
  X.rT = X.scale ? __fdiv_rn(1.0f, X.T) : 1.0f;
  sA = X.scale ? X.rT : 1.0f;
  X.A2 = CFG ? __fmul_rn(__fmul_rn(kLog2e, P.cfg_1pw), sA) : __fmul_rn(kLog2e, sA);
  X.B2 = CFG ? __fmul_rn(__fmul_rn(kLog2e, P.cfg_w), sA) : 0.f;
}

// Group maxima m[] and sums s[] (relative to m*scale) -> the position context
// (stats_core: maxima, sums, z2 offset) and the scoring context (stats_rest).
// The group and its tail warp both derive them here, so the two see
// identical values.
template <bool CFG>
__device__ __forceinline__ void stats_core(const float (&m)[3], const float (&s)[3], PosCtx& X) {
  const float kPosInf = __int_as_float(0x7f800000);
  const float kNaN = __int_as_float(0x7fc00000);
  X.mc = m[0];
  X.mu = CFG ? m[1] : 0.f;
  X.Sc = (X.mc > kNegInf && X.mc < kPosInf) ? s[0] : kNaN;
  X.Su = CFG ? ((X.mu > kNegInf && X.mu < kPosInf) ? s[1] : kNaN) : 0.f;
  X.K2 = CFG ? __fmaf_rn(-X.mc, X.A2, __fmul_rn(X.mu, X.B2)) : __fmul_rn(-X.mc, X.A2);
  X.zmax = __fadd_rn(m[2], X.K2);
  X.S = (m[2] < kPosInf && s[2] < kPosInf) ? s[2] : kNaN;
}

// The rest of the contexts (logs and reciprocals), for exact values and scores.
template <bool CFG>
__device__ __forceinline__ void stats_rest(const SampleParams& P, const ItemParams& Q, float sA, PosCtx& X,
                                           ScoreCtx& K) {
  X.lc = logf(X.Sc);
  X.lu = CFG ? logf(X.Su) : 0.f;
  X.Kval = CFG ? __fmul_rn(__fsub_rn(__fmul_rn(P.cfg_w, X.lu), __fmul_rn(P.cfg_1pw, X.lc)), sA)
               : __fmul_rn(X.mc, sA);
  const bool topk_on = Q.top_k > 0 && Q.top_k < P.V;
  const bool pen_on = P.history_kind != YAPD_HISTORY_NONE && P.history != nullptr && Q.rep != 1.0f;
  K.b = Q.pos / P.L;
  K.pos = Q.pos;
  K.l = Q.pos - K.b * P.L;
  K.pen_on = pen_on;
  K.noisy = X.T > 0.0f || !P.zero_temp_greedy;
  K.turbo = topk_on || Q.top_p < 1.0f || Q.min_p > 0.0f || K.pen_on;
  K.minp_on = false;
  K.rep = Q.rep;
  K.rrep = K.pen_on ? __fdiv_rn(1.0f, Q.rep) : 1.0f;
  K.r = __fdiv_rn(1.0f, X.S);
  K.minp_thr = 0.f;
  K.hbits = nullptr;
}

// The min-p band's ids, from the vectors pass 2 marked (and every scalar
// element), into the stage's hand-off record (the first 32 of them); returns
// the band size.  h.n must be zero on entry.
template <class C, bool CFG>
__device__ __forceinline__ int band_collect(const PosCtx& X, const RowRef<C>& R, const Span& S, uint32_t marks,
                                            float lo_z, Hand& h) {
  const int tid = gtid<C>();
  while (marks) {
    const int k = __ffs(marks) - 1;
    marks &= marks - 1u;
    const int j = S.j0 + tid + k * C::NT;
    const uint4 a = lds128(R.sc + j * 16);
    uint4 q = a;
    if (CFG) q = lds128(R.su + j * 16);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      const float z = z2_of(X, velem<C>(a, i), CFG ? velem<C>(q, i) : 0.f);
      m |= (z >= lo_z ? 1u : 0u) << i;
    }
    const int v0 = j * C::W - S.head;
    while (m) {
      const int i = __ffs(m) - 1;
      m &= m - 1u;
      const int at = atomicAdd(&h.n, 1);
      if (at < 32) h.cv[at] = v0 + i;
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    if (z2_smem<C>(X, R, v) >= lo_z) {
      const int at = atomicAdd(&h.n, 1);
      if (at < 32) h.cv[at] = v;
    }
  }
  csync<C>();
  return h.n;
}

// ------------------------------------------------------------ histogram select
//
// Positions filtered by top-k and / or top-p (min-p off) take three passes
// over their staged rows:
//   1. the exact maxima of c, u and z2' = A2*c - B2*u;
//   2. the sums of exp(c - max c), exp(u - max u) and 2^d, d = z2 - zmax,
//      against those maxima, and a histogram of d by depth below zmax
//      (kHistBins bins of 1/kHistPerUnit log2 unit: counts and fixed-point
//      masses 2^d by shared-memory integer atomics).  One warp scans it for
//      the bin where the count from the top reaches k, and the bins where the
//      mass from the top reaches top_p times the bounds of S_k (the top-k
//      mass) that bin gives, and lays out the bands;
//   3. one collection pass: tokens of the crossing bins, widened by the float
//      margin, go to the band lists with their exact values and masses;
//      tokens above the top band (all kept) go to the kept list with their
//      masses summed; tokens between the bands are not visited (their count
//      and mass come from the histogram).
// The kept tokens are then scored exactly (penalty, Philox noise), one per
// thread; the bands are resolved as select_cold resolves its bands (rank by
// (exact value, id), the top-k cut and S_k, top-p flags from double prefix
// sums), their kept members are scored, and the best score wins.  On a
// failed precondition (non-finite row, a crossing below the binned range, a
// band larger than the list, a crossing the histogram misplaced) the function
// writes nothing and returns false; the caller then takes the general cold
// path.

constexpr int kHistPerUnit = 8;  // kHistBins / kHistPerUnit = 64 log2 units of depth

// Group maxima of three values (one barrier).
template <class C>
__device__ __forceinline__ void red_max3(float& a, float& b, float& c, Smem<C>& sm, int& slot) {
  a = warp_max(a);
  b = warp_max(b);
  c = warp_max(c);
  float* s = sm.red8 + slot * 8 * C::NW;
  slot ^= 1;
  if ((threadIdx.x & 31) == 0) {
    s[gtid<C>() >> 5] = a;
    s[C::NW + (gtid<C>() >> 5)] = b;
    s[2 * C::NW + (gtid<C>() >> 5)] = c;
  }
  csync<C>();
  float ra = s[0], rb = s[C::NW], rc = s[2 * C::NW];
#pragma unroll
  for (int q = 1; q < C::NW; ++q) {
    ra = fmaxf(ra, s[q]);
    rb = fmaxf(rb, s[C::NW + q]);
    rc = fmaxf(rc, s[2 * C::NW + q]);
  }
  a = ra;
  b = rb;
  c = rc;
}

// Pass 1: this thread's maxima of c, u and z2' = A2*c - B2*u (NaN ignored).
template <class C, bool CFG>
__device__ __forceinline__ void hpass_max(const PosCtx& X, const RowRef<C>& R, const Span& S, float& mc, float& mu,
                                          float& zm) {
  const int tid = gtid<C>();
  const float A2 = X.A2, nB2 = -X.B2;
  float z0 = kNegInf, z1 = kNegInf;
  if constexpr (C::BF16) {
    uint32_t c2 = 0xff80ff80u, u2 = 0xff80ff80u;
    const unsigned long long A2p = f2_pack(A2, A2), nB2p = f2_pack(nB2, nB2), zp = f2_pack(0.f, 0.f);
#pragma unroll 1
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      c2 = bmax2(c2, bmax2(bmax2(a.x, a.y), bmax2(a.z, a.w)));
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      uint32_t qw[4] = {0u, 0u, 0u, 0u};
      if (CFG) {
        const uint4 q = lds128(R.su + j * 16);
        u2 = bmax2(u2, bmax2(bmax2(q.x, q.y), bmax2(q.z, q.w)));
        qw[0] = q.x;
        qw[1] = q.y;
        qw[2] = q.z;
        qw[3] = q.w;
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const unsigned long long cx = f2_bf16(aw[t]);
        const unsigned long long zx = CFG ? f2_fma(cx, A2p, f2_fma(f2_bf16(qw[t]), nB2p, zp)) : f2_fma(cx, A2p, zp);
        float lo, hi;
        f2_unpack(zx, lo, hi);
        if (t & 1) z1 = fmax3(z1, lo, hi);
        else z0 = fmax3(z0, lo, hi);
      }
    }
    mc = fmaxf(bf16lo(c2), bf16hi(c2));
    mu = CFG ? fmaxf(bf16lo(u2), bf16hi(u2)) : kNegInf;
  } else {
    float c0 = kNegInf, u0 = kNegInf;
#pragma unroll 2
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      const float cv[4] = {__uint_as_float(a.x), __uint_as_float(a.y), __uint_as_float(a.z), __uint_as_float(a.w)};
      c0 = fmax3(c0, cv[0], cv[1]);
      c0 = fmax3(c0, cv[2], cv[3]);
      float zz[4];
      if (CFG) {
        const uint4 q = lds128(R.su + j * 16);
        const float uv[4] = {__uint_as_float(q.x), __uint_as_float(q.y), __uint_as_float(q.z), __uint_as_float(q.w)};
        u0 = fmax3(u0, uv[0], uv[1]);
        u0 = fmax3(u0, uv[2], uv[3]);
#pragma unroll
        for (int i = 0; i < 4; ++i) zz[i] = __fmaf_rn(cv[i], A2, __fmul_rn(uv[i], nB2));
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) zz[i] = __fmul_rn(cv[i], A2);
      }
      z0 = fmax3(z0, zz[0], zz[1]);
      z1 = fmax3(z1, zz[2], zz[3]);
    }
    mc = c0;
    mu = CFG ? u0 : kNegInf;
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    mc = fmaxf(mc, c);
    float z;
    if (CFG) {
      const float u = load_elem_smem<C>(R.su, R.gu, v);
      mu = fmaxf(mu, u);
      z = __fmaf_rn(c, A2, __fmul_rn(u, nB2));
    } else {
      z = __fmul_rn(c, A2);
    }
    z0 = fmaxf(z0, z);
  }
  zm = fmaxf(z0, z1);
}

// d = z2 - zmax of one token (the histogram select's key), from its logits.
template <bool CFG>
__device__ __forceinline__ float hdepth(const PosCtx& X, float K2mz, float c, float u) {
  return CFG ? __fmaf_rn(c, X.A2, __fmaf_rn(u, -X.B2, K2mz)) : __fmaf_rn(c, X.A2, K2mz);
}

// Exact scores of every kept token (depth d >= dH) of the staged rows into
// `kb`.  Each warp takes its lanes' vectors together: the lanes' kept tokens,
// grouped by Philox block, go to the warp's queue in shared memory (sm.kq),
// and the lanes then score the queued blocks round-robin, so that a warp
// spends one scoring slot per 32 kept blocks instead of one per token of a
// vector that any lane keeps.  Tokens of one block share its Philox word
// set, and a token whose noise cannot lift it to the best score known (the
// warp's best so far, or `thr`, the score of a token the group has already
// scored) skips the logarithms: the Gumbel noise obeys G = -ln(-ln u) <=
// -ln(1 - u) (as -ln u >= 1 - u), so with s0 its exact score before the
// noise, s0 + G < best - tiny whenever 1 - u > e^-(best - tiny - s0); `tiny`
// covers the rounding of s0 + G, and such a token scores strictly below a
// token already scored, whatever the tie rule.
template <class C, bool CFG>
__device__ __forceinline__ void kept_pass(const SampleParams& P, const PosCtx& X, const ScoreCtx& K,
                                          const RowRef<C>& R, const Span& S, float K2mz, float dH, Pick& kb,
                                          Smem<C>& sm, float thr) {
  const bool philox = K.noisy && P.noise_kind != YAPD_NOISE_EXPLICIT;
  const int lane = threadIdx.x & 31;
  uint32_t* q = sm.kq + (gtid<C>() >> 5) * kKqPerWarp;
  float best = kb.score > thr ? kb.score : thr;
  // the kept tokens v4 + i (bit i of keep) of one Philox block
  auto unit = [&](int v4, unsigned keep) {
    Philox4 r{0u, 0u, 0u, 0u};
    if (philox)
      r = philox4x32_10((uint32_t)v4 >> 2, (uint32_t)K.pos, (uint32_t)P.offset,
                        (uint32_t)(P.offset >> 32) & 0x7fffffffu, (uint32_t)P.seed, (uint32_t)(P.seed >> 32));
    while (keep) {
      const int i = __ffs(keep) - 1;
      keep &= keep - 1u;
      const int v = v4 + i;
      const float c = load_elem_smem<C>(R.sc, R.gc, v);
      const float u = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
      const float vals = exact_val_cu(P, X, c, u);
      const bool hb = K.pen_on ? hist_bit_k(P, K, v) : false;
      const float s0 = (K.pen_on && hb) ? penalize(vals, K.rep, K.rrep) : vals;
      float es = s0;
      if (philox) {
        const float uu = uniform_from_word(philox_word(r, (uint32_t)i));
        if (best > kNegInf && best < __int_as_float(0x7f800000)) {
          const float t = best - (1e-6f * fabsf(best) + 1e-6f) - s0;
          if (t > 0.0f) {
            const float qb = ex2_approx(-t * kLog2e) * 1.0001f;  // e^-t, rounded up past ex2.approx's error
            if (__fsub_rn(1.0f, uu) > qb) continue;
          }
        }
        es = __fadd_rn(s0, gumbel_from_uniform(uu));
      } else if (K.noisy) {
        es = __fadd_rn(s0, noise_at(P, K.b, K.pos, K.l, v));
      }
      const Pick cand{es, vals, v};
      if (es == es && es > kNegInf && pick_better(cand, kb, K.turbo)) {
        kb = cand;
        best = fmaxf(best, es);
      }
    }
  };
  const int nk = (S.j1 - S.j0 + C::NT - 1) / C::NT;
  for (int k = 0; k < nk; ++k) {
    const int j = S.j0 + gtid<C>() + k * C::NT;
    // this lane's kept tokens of vector j, as (block, mask) units
    uint32_t un[3] = {0u, 0u, 0u};
    int nu = 0;
    if (j < S.j1) {
      const uint4 a = lds128(R.sc + j * 16);
      const uint4 bq = CFG ? lds128(R.su + j * 16) : a;
      const int v0 = j * C::W - S.head;
      unsigned m = 0u;
#pragma unroll
      for (int i = 0; i < C::W; ++i)
        m |= (hdepth<CFG>(X, K2mz, velem<C>(a, i), CFG ? velem<C>(bq, i) : 0.f) >= dH ? 1u : 0u) << i;
#pragma unroll
      for (int t = 0; t < 3; ++t) {
        if (m) {
          const int i = __ffs(m) - 1;
          const int v4 = (v0 + i) & ~3;
          const int i0 = v4 - v0;  // -3..W-1: bit of token v4 in m
          const unsigned blk = i0 >= 0 ? (m >> i0) & 15u : (m << (-i0)) & 15u;
          m &= i0 >= 0 ? ~(15u << i0) : ~(15u >> (-i0));
          un[t] = ((uint32_t)v4 << 4) | blk;
          ++nu;
        }
      }
    }
    int incl = nu;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    if (total == 0) continue;
#pragma unroll
    for (int t = 0; t < 3; ++t)
      if (t < nu) q[incl - nu + t] = un[t];
    __syncwarp();
    for (int t = lane; t < total; t += 32) {
      const uint32_t e = q[t];
      unit((int)(e >> 4), e & 15u);
    }
    best = warp_max(best);
    __syncwarp();
  }
  for (int e = gtid<C>(); e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    const float u = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
    if (hdepth<CFG>(X, K2mz, c, u) >= dH) unit(v & ~3, 1u << (v & 3));
  }
}

// Histogram bin of a depth d <= 0: j = rint(-kHistPerUnit * d), so bin j
// holds d in (-(j + 1/2) / kHistPerUnit, -(j - 1/2) / kHistPerUnit]; -1 past
// the binned range (and for non-finite d).  Rounding by the 1.5 * 2^23 shift
// keeps the float-to-integer conversion off the conversion pipe.
__device__ __forceinline__ int hist_bin(float d) {
  const int j = __float_as_int(__fadd_rn(__fmul_rn(d, -(float)kHistPerUnit), 12582912.0f)) - 0x4B400000;
  return j < kHistBins ? max(j, 0) : -1;
}

// A token's mass 2^d in the histogram's fixed point: rint(e * 2^(16 + o))
// with o = j / kHistPerUnit its octave of depth, so that every member of a
// bin weighs about 2^16 units (the scale is an exponent add, exact).  Shared
// memory has no native float atomic add; two integer atomics per token cost
// a third of one float atomic.
__device__ __forceinline__ uint32_t hist_q(float e, int j) {
  const float t = __int_as_float(__float_as_int(e) + ((16 + j / kHistPerUnit) << 23));
  return (uint32_t)(__float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000);
}
__device__ __forceinline__ float hist_mass(uint32_t q, int j) {
  return __fmul_rn((float)q, __int_as_float((127 - 16 - j / kHistPerUnit) << 23));
}

template <class C>
__device__ __forceinline__ void hist_add(Smem<C>& sm, float d, float e) {
  const int j = hist_bin(d);
  if (j >= 0) {
    atomicAdd(&sm.hc[j], 1);
    atomicAdd(&sm.hq[j], hist_q(e, j));
  }
}

// Pass 2: sums against the group maxima and the depth histogram.
template <class C, bool CFG>
__device__ __forceinline__ void hpass_sums(const PosCtx& X, const RowRef<C>& R, const Span& S, float K2mz,
                                           float& sc, float& su, float& s, Smem<C>& sm) {
  const int tid = gtid<C>();
  const float nmcL = -__fmul_rn(X.mc, kLog2e), nmuL = CFG ? -__fmul_rn(X.mu, kLog2e) : 0.f;
  float sc0 = 0.f, sc1 = 0.f, su0 = 0.f, su1 = 0.f, s0 = 0.f, s1 = 0.f;
  if constexpr (C::BF16) {
    const unsigned long long L2p = f2_pack(kLog2e, kLog2e), A2p = f2_pack(X.A2, X.A2),
                             nB2p = f2_pack(-X.B2, -X.B2), Kp = f2_pack(K2mz, K2mz);
    const unsigned long long nmcLp = f2_pack(nmcL, nmcL), nmuLp = f2_pack(nmuL, nmuL);
    unsigned long long scp = f2_pack(0.f, 0.f), sup = scp, sp = scp;
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      uint4 q = a;
      if (CFG) q = lds128(R.su + j * 16);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const unsigned long long cx = f2_bf16(aw[t]);
        unsigned long long dx;
        float lo, hi;
        if (CFG) {
          const unsigned long long ux = f2_bf16(qw[t]);
          dx = f2_fma(cx, A2p, f2_fma(ux, nB2p, Kp));
          f2_unpack(f2_fma(ux, L2p, nmuLp), lo, hi);
          sup = f2_add(sup, f2_pack(ex2_approx(lo), ex2_approx(hi)));
        } else {
          dx = f2_fma(cx, A2p, Kp);
        }
        f2_unpack(f2_fma(cx, L2p, nmcLp), lo, hi);
        scp = f2_add(scp, f2_pack(ex2_approx(lo), ex2_approx(hi)));
        f2_unpack(dx, lo, hi);
        const float elo = ex2_approx(lo), ehi = ex2_approx(hi);
        sp = f2_add(sp, f2_pack(elo, ehi));
        hist_add<C>(sm, lo, elo);
        hist_add<C>(sm, hi, ehi);
      }
    }
    f2_unpack(scp, sc0, sc1);
    f2_unpack(sup, su0, su1);
    f2_unpack(sp, s0, s1);
  } else {
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      uint4 q = a;
      if (CFG) q = lds128(R.su + j * 16);
#pragma unroll
      for (int i = 0; i < C::W; ++i) {
        const float c = velem<C>(a, i);
        const float u = CFG ? velem<C>(q, i) : 0.f;
        const float d = hdepth<CFG>(X, K2mz, c, u);
        const float e = ex2_approx(d);
        if (i & 1) {
          sc1 += ex2_approx(__fmaf_rn(c, kLog2e, nmcL));
          if (CFG) su1 += ex2_approx(__fmaf_rn(u, kLog2e, nmuL));
          s1 += e;
        } else {
          sc0 += ex2_approx(__fmaf_rn(c, kLog2e, nmcL));
          if (CFG) su0 += ex2_approx(__fmaf_rn(u, kLog2e, nmuL));
          s0 += e;
        }
        hist_add<C>(sm, d, e);
      }
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    const float u = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
    sc0 += ex2_approx(__fmaf_rn(c, kLog2e, nmcL));
    if (CFG) su0 += ex2_approx(__fmaf_rn(u, kLog2e, nmuL));
    const float d = hdepth<CFG>(X, K2mz, c, u);
    const float ed = ex2_approx(d);
    s0 += ed;
    hist_add<C>(sm, d, ed);
  }
  sc = sc0 + sc1;
  su = su0 + su1;
  s = s0 + s1;
}

// The scan (the group's first warp).  The bins are taken 128 at a time, bin 0
// (the top) first, lane l holding bins 128 q + 4 l + (0..3) of block q, with
// warp prefix sums carried from block to block; each search stops at the
// first block that holds its crossing (the crossings usually lie in the first
// block).  Finds the bin jk where the count from the top reaches k, the bins
// jp1 <= jp2 where the mass from the top reaches the lower / upper top-p
// target (top_p times the bounds of S_k that bin jk gives, or times S_all),
// and lays out the bands: band P = bins [ja, jb] (the top-p crossing, merged
// with jk when they touch; jk alone without top-p) and, when jk lies further
// down, band K = bin jk with the bins between them summed.
// sm.hsi: [0] ok, [1] ja, [2] jb, [3] jk, [4] sep, [5] count between;
// sm.hsf: [0] mass between.
template <class C>
__device__ __forceinline__ void hist_scan(Smem<C>& sm, bool topk_on, int k, bool topp_on, float top_p, float S_all) {
  constexpr int NBLK = kHistBins / 128;
  const unsigned full = 0xffffffffu;
  const int lane = threadIdx.x & 31;
  // block q: this lane's running bin masses from the top of its four (lm),
  // and the block's mass before this lane (em) and through it (im)
  auto blk_mass = [&](int q, float (&lm)[4], float& em, float& im) {
    const int j0 = q * 128 + 4 * lane;
    const uint4 m4 = *reinterpret_cast<const uint4*>(sm.hq + j0);
    lm[0] = hist_mass(m4.x, j0);
    lm[1] = lm[0] + hist_mass(m4.y, j0 + 1);
    lm[2] = lm[1] + hist_mass(m4.z, j0 + 2);
    lm[3] = lm[2] + hist_mass(m4.w, j0 + 3);
    im = lm[3];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(full, im, o);
      if (lane >= o) im += y;
    }
    em = __shfl_up_sync(full, im, 1);
    if (lane == 0) em = 0.f;
  };
  bool ok = true;
  int jk = -1;
  float slo = S_all, shi = S_all;
  if (topk_on) {
    int cbase = 0;
    float mbase = 0.f;
#pragma unroll 1
    for (int q = 0; q < NBLK; ++q) {
      const int j0 = q * 128 + 4 * lane;
      const int4 c4 = *reinterpret_cast<const int4*>(sm.hc + j0);
      const int lc[4] = {c4.x, c4.x + c4.y, c4.x + c4.y + c4.z, c4.x + c4.y + c4.z + c4.w};
      int ic = lc[3];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(full, ic, o);
        if (lane >= o) ic += y;
      }
      const int ec = cbase + ic - lc[3];
      float lm[4], em, im;
      blk_mass(q, lm, em, im);
      const unsigned bk = __ballot_sync(full, cbase + ic >= k);
      if (bk) {
        const int sl = __ffs(bk) - 1;
        int i = 3;
        if (ec + lc[2] >= k) i = 2;
        if (ec + lc[1] >= k) i = 1;
        if (ec + lc[0] >= k) i = 0;
        const float before = __fadd_rn(mbase, em);
        const float lmi = i == 0 ? lm[0] : i == 1 ? lm[1] : i == 2 ? lm[2] : lm[3];
        const float lmp = i == 1 ? lm[0] : i == 2 ? lm[1] : lm[2];
        const float lo = i == 0 ? before : __fadd_rn(before, lmp);
        const float hi = __fadd_rn(before, lmi);
        jk = q * 128 + 4 * sl + __shfl_sync(full, i, sl);
        slo = __shfl_sync(full, lo, sl);
        shi = __shfl_sync(full, hi, sl);
        break;
      }
      cbase += __shfl_sync(full, ic, 31);
      mbase += __shfl_sync(full, im, 31);
    }
    if (jk < 0) ok = false;  // the k-th token lies below the binned range
  }
  int ja = jk, jb = jk;
  if (ok && topp_on) {
    // the fixed-point masses are exact to about 2^-16 per token: 1e-4 slack
    const float tlo = __fmul_rn(__fmul_rn(top_p, slo), 0.9999f);
    const float thi = __fmul_rn(__fmul_rn(top_p, shi), 1.0001f);
    // with top-k the cut never lies below the k-th token: blocks past jk's
    // could only clamp to jk (and tlo < slo is always reached before it)
    const int qlast = topk_on ? (jk >> 7) : NBLK - 1;
    int a1 = -1, a2 = -1;
    float mbase = 0.f;
    // the first bin of block q whose running mass reaches t (lane sl is the
    // first lane whose four bins reach it)
    auto first_at = [&](int q, const float (&lm)[4], float before, float t, unsigned bal) {
      const int sl = __ffs(bal) - 1;
      int i = 3;
      if (__fadd_rn(before, lm[2]) >= t) i = 2;
      if (__fadd_rn(before, lm[1]) >= t) i = 1;
      if (__fadd_rn(before, lm[0]) >= t) i = 0;
      return q * 128 + 4 * sl + __shfl_sync(full, i, sl);
    };
#pragma unroll 1
    for (int q = 0; q <= qlast; ++q) {
      float lm[4], em, im;
      blk_mass(q, lm, em, im);
      const float before = __fadd_rn(mbase, em);
      const float end = __fadd_rn(before, lm[3]);
      if (a1 < 0) {
        const unsigned b1 = __ballot_sync(full, end >= tlo);
        if (b1) a1 = first_at(q, lm, before, tlo, b1);
      }
      const unsigned b2 = __ballot_sync(full, end >= thi);
      if (b2) {
        a2 = first_at(q, lm, before, thi, b2);
        break;
      }
      mbase += __shfl_sync(full, im, 31);
    }
    if (a1 < 0) {
      if (topk_on) a1 = jk;
      else ok = false;
    }
    ja = a1;
    jb = a2;
    if (topk_on) {
      if (jb < 0 || jb > jk) jb = jk;
      if (ja > jk) ja = jk;
    } else if (jb < 0) {
      ok = false;
    }
  }
  const bool sep = ok && topp_on && topk_on && jk > jb + 1;
  if (ok && topp_on && topk_on && !sep) jb = jk;
  // tokens of the bins strictly between band P and band K
  int nbt = 0;
  float mbt = 0.f;
  if (sep) {
#pragma unroll 1
    for (int q = (jb + 1) >> 7; q <= ((jk - 1) >> 7); ++q) {
      const int j0 = q * 128 + 4 * lane;
      const int4 c4 = *reinterpret_cast<const int4*>(sm.hc + j0);
      const uint4 m4 = *reinterpret_cast<const uint4*>(sm.hq + j0);
      const int cc[4] = {c4.x, c4.y, c4.z, c4.w};
      const uint32_t mq[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = j0 + i;
        if (j > jb && j < jk) {
          nbt += cc[i];
          mbt += hist_mass(mq[i], j);
        }
      }
    }
    nbt = warp_sum_i(nbt);
    mbt = warp_sum(mbt);
  }
  if (lane == 0) {
    sm.hsi[0] = ok ? 1 : 0;
    sm.hsi[1] = ja;
    sm.hsi[2] = jb;
    sm.hsi[3] = jk;
    sm.hsi[4] = sep ? 1 : 0;
    sm.hsi[5] = nbt;
    sm.hsf[0] = mbt;
    sm.misc[0] = 0;  // band and kept-list counters of pass 3
    sm.misc[1] = 0;
    sm.misc[2] = 0;
  }
}

template <class C, bool CFG>
__device__ __noinline__ bool select_hist(const SampleParams& P, const ItemParams Q, const RowRef<C> R, const Span S,
                                         Smem<C>& sm, Hand& hd) {
  csync<C>();  // out-of-line reductions use scratch slots 2/3
  int slot = 2;
  const int tid = gtid<C>();
  const int V = P.V;
  const float kPosInf = __int_as_float(0x7f800000);
  const bool topk_on = Q.top_k > 0 && Q.top_k < V;
  const bool topp_on = Q.top_p < 1.0f;
  PosCtx X;
  float sA;
  item_ctx<CFG>(P, Q, X, sA);
  for (int i = tid; i < kHistBins; i += C::NT) {
    sm.hc[i] = 0;
    sm.hq[i] = 0u;
  }
  // ---- pass 1: group maxima ----
  float mc, mu, zm;
  hpass_max<C, CFG>(X, R, S, mc, mu, zm);
  red_max3<C>(mc, mu, zm, sm, slot);
  if (!(mc > kNegInf && mc < kPosInf) || (CFG && !(mu > kNegInf && mu < kPosInf)) ||
      !(zm > kNegInf && zm < kPosInf))
    return false;
  // ---- pass 2: sums and the depth histogram ----
  X.mc = mc;
  X.mu = CFG ? mu : 0.f;
  X.K2 = CFG ? __fmaf_rn(-mc, X.A2, __fmul_rn(mu, X.B2)) : __fmul_rn(-mc, X.A2);
  const float zmax = __fadd_rn(zm, X.K2);
  const float K2mz = __fsub_rn(X.K2, zmax);
  float sums[8];
  hpass_sums<C, CFG>(X, R, S, K2mz, sums[0], sums[1], sums[2], sm);
#pragma unroll
  for (int j = 3; j < 8; ++j) sums[j] = 0.f;
  block_sum8<C>(sums, sm, slot);
  {
    const float m3[3] = {mc, CFG ? mu : kNegInf, zm};
    const float s3[3] = {sums[0], sums[1], sums[2]};
    stats_core<CFG>(m3, s3, X);
  }
  if (!(X.Sc == X.Sc) || !(X.Sc > 0.f) || (CFG && !(X.Su == X.Su && X.Su > 0.f)) || !(X.S == X.S) ||
      !(X.S > 0.f))
    return false;
  ScoreCtx K;
  stats_rest<CFG>(P, Q, sA, X, K);
  // ---- the scan ----
  if (tid < 32) hist_scan<C>(sm, topk_on, Q.top_k, topp_on, Q.top_p, X.S);
  csync<C>();
  if (!sm.hsi[0]) return false;
  const int ja = sm.hsi[1], jb = sm.hsi[2], jk = sm.hsi[3];
  const bool sep = sm.hsi[4] != 0;
  const float n_bins_between = (float)sm.hsi[5];
  const float m_bins_between = sm.hsf[0];
  // bin edges in d, widened by the float margin of z2 against the exact values
  auto edge = [&](float jh, bool upper) {
    const float d = __fmul_rn(-jh, 1.0f / (float)kHistPerUnit);
    const float m = zmargin(__fadd_rn(zmax, d));
    return upper ? __fadd_rn(d, m) : __fsub_rn(d, m);
  };
  const float dH = edge((float)ja - 0.5f, true);     // above band P: kept
  const float dPl = edge((float)jb + 0.5f, false);   // band P: [dPl, dH)
  const float dKh = sep ? edge((float)jk - 0.5f, true) : dPl;
  const float dKl = sep ? edge((float)jk + 0.5f, false) : dPl;  // band K: [dKl, dKh)
  // ---- pass 3: the bands, the kept set's candidates ----
  // (tokens between the bands are not visited: their count and mass come from
  // the histogram, less the band members that sit in those bins)
  float n_above = 0.f, m_above = 0.f, m_bandP = 0.f, n_corr = 0.f, m_corr = 0.f, m_bandK = 0.f;
  auto visit = [&](int v) {
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    const float u = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
    const float d = hdepth<CFG>(X, K2mz, c, u);
    const float e = ex2_approx(d);
    if (d >= dH) {
      // kept: scored after the pass, one token per thread
      n_above += 1.f;
      m_above += e;
      const int at = atomicAdd(&sm.misc[2], 1);
      if (at < C::NT) sm.klist[at] = v;
      return;
    }
    const bool inP = d >= dPl;
    if (!inP && !(d >= dKl && d < dKh)) return;
    if (sep) {
      // members in the bins strictly between the bands
      const int j = hist_bin(d);
      if (j > jb && j < jk) {
        n_corr += 1.f;
        m_corr += e;
      }
    }
    if (inP) {
      m_bandP += e;
      const int at = atomicAdd(&sm.misc[0], 1);
      if (at < C::BAND) {
        sm.cand[at] = cand_key(exact_val_cu(P, X, c, u), v);
        sm.cande[at] = e;
      }
    } else {
      m_bandK += e;
      const int at = atomicAdd(&sm.misc[1], 1);
      const int idx = C::BAND - 1 - at;
      if (idx >= 0) {
        sm.cand[idx] = cand_key(exact_val_cu(P, X, c, u), v);
        sm.cande[idx] = e;
      }
    }
  };
  // d in band K <=> |d - cK| < hK (never true without band K)
  const float cK = __fmul_rn(0.5f, __fadd_rn(dKl, dKh)), hK = sep ? __fmul_rn(0.5f, __fsub_rn(dKh, dKl)) : -1.f;
  auto wanted = [&](float d) { return d >= dPl || fabsf(__fsub_rn(d, cK)) <= hK; };
  if constexpr (C::BF16) {
    const unsigned long long A2p = f2_pack(X.A2, X.A2), nB2p = f2_pack(-X.B2, -X.B2), Kp = f2_pack(K2mz, K2mz);
    const float dLow = sep ? dKl : dPl;
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      uint4 q = a;
      if (CFG) q = lds128(R.su + j * 16);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
      float dd[8];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const unsigned long long cx = f2_bf16(aw[t]);
        const unsigned long long dx = CFG ? f2_fma(cx, A2p, f2_fma(f2_bf16(qw[t]), nB2p, Kp)) : f2_fma(cx, A2p, Kp);
        f2_unpack(dx, dd[2 * t], dd[2 * t + 1]);
      }
      const float vm = fmaxf(fmax3(fmax3(dd[0], dd[1], dd[2]), dd[3], dd[4]), fmax3(dd[5], dd[6], dd[7]));
      if (!(vm >= dLow)) continue;
      uint32_t m = 0u;
#pragma unroll
      for (int i = 0; i < 8; ++i) m |= (wanted(dd[i]) ? 1u : 0u) << i;
      const int v0 = j * C::W - S.head;
      while (m) {
        const int i = __ffs(m) - 1;
        m &= m - 1u;
        visit(v0 + i);
      }
    }
  } else {
    for (int j = S.j0 + tid; j < S.j1; j += C::NT) {
      const uint4 a = lds128(R.sc + j * 16);
      uint4 q = a;
      if (CFG) q = lds128(R.su + j * 16);
      uint32_t m = 0u;
#pragma unroll
      for (int i = 0; i < C::W; ++i) {
        const float d = hdepth<CFG>(X, K2mz, velem<C>(a, i), CFG ? velem<C>(q, i) : 0.f);
        m |= (wanted(d) ? 1u : 0u) << i;
      }
      const int v0 = j * C::W - S.head;
      while (m) {
        const int i = __ffs(m) - 1;
        m &= m - 1u;
        visit(v0 + i);
      }
    }
  }
  for (int e = tid; e < S.nscal; e += C::NT) {
    const int v = scalar_v(S, e);
    const float c = load_elem_smem<C>(R.sc, R.gc, v);
    const float u = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
    if (wanted(hdepth<CFG>(X, K2mz, c, u))) visit(v);
  }
  float acc[8] = {n_above, m_above, m_bandP, n_corr, m_corr, m_bandK, 0.f, 0.f};
  block_sum8<C>(acc, sm, slot);
  m_bandK = acc[5];
  n_above = acc[0];
  m_above = acc[1];
  m_bandP = acc[2];
  const float n_between = n_bins_between - acc[3];
  const float m_between = __fsub_rn(m_bins_between, acc[4]);
  const int nP = sm.misc[0], nK = sm.misc[1], nA = sm.misc[2];
  if (nP + nK > C::BAND || nP == 0 || (sep && nK == 0)) return false;
  // ---- hand the rest to the group's tail warp ----
  // (top-p rows whose lists fit the hand-off record, when the float bounds of
  // S_k already guarantee what the exact resolution checks: band P's first
  // member kept, every token below band P dropped, the k-th token in band K)
  {
    bool hand = topp_on && nP <= 32 && (!topk_on || sep);
    float s_lo = X.S, s_hi = X.S;
    bool sk_exact = false;
    if (hand && sep) {
      const int kl = Q.top_k - (int)(n_above + (float)nP + n_between);
      s_lo = __fadd_rn(__fadd_rn(m_above, m_bandP), fmaxf(m_between, 0.f));
      s_hi = __fadd_rn(s_lo, m_bandK);
      hand = kl >= 1 && kl <= nK;
      if (hand && nK > 32) {
        // band K too large for the tail warp's lanes: S_k here, exactly as
        // the resolution below computes it (rank by (exact value, id))
        float part = 0.f;
        for (int q = tid; q < nK; q += C::NT) {
          const unsigned long long key = sm.cand[C::BAND - 1 - q];
          int rank = 0;
          for (int j2 = 0; j2 < nK; ++j2) rank += (sm.cand[C::BAND - 1 - j2] > key) ? 1 : 0;
          if (rank < kl) part += sm.cande[C::BAND - 1 - q];
        }
        s_lo = __fadd_rn(s_lo, block_sum1<C>(part, sm, slot));
        s_hi = s_lo;
        sk_exact = true;
      }
    }
    hand = hand && m_above < __fmul_rn(__fmul_rn(Q.top_p, s_lo), 0.99999f) &&
           __fadd_rn(m_above, m_bandP) >= __fmul_rn(__fmul_rn(Q.top_p, s_hi), 1.00001f);
    if (hand) {
      // the kept set: its ids for the tail, or (too many) its best scored here
      int best_kept = -1;
      if (nA > 64) {
        Pick kb{kNegInf, kNegInf, 0x7fffffff};
        for (int q = tid; q < nA && q < C::NT; q += C::NT) {
          const int v = sm.klist[q];
          const float vals = exact_val<C>(P, X, R, v);
          const float es = exact_score<C>(P, K, v, vals);
          const Pick cand{es, vals, v};
          if (es == es && es > kNegInf && pick_better(cand, kb, K.turbo)) kb = cand;
        }
        if (nA > C::NT) {
          // more kept tokens than the list holds: all of them, against the
          // best score of the listed ones
          const float thr = red_max1<C>(kb.score, sm, slot);
          kept_pass<C, CFG>(P, X, K, R, S, K2mz, dH, kb, sm, thr);
        }
        best_kept = block_pick<C>(kb, K.turbo, sm, slot);
      }
      if (tid < nP) hd.pid[tid] = cand_id(sm.cand[tid]);
      if (!sk_exact && tid < nK) hd.kid[tid] = cand_id(sm.cand[C::BAND - 1 - tid]);
      if (nA <= 64 && tid < nA) hd.aid[tid] = sm.klist[tid];
      if (tid == 0) {
        hd.m[0] = X.mc;
        hd.m[1] = CFG ? X.mu : kNegInf;
        hd.m[2] = zm;
        hd.s[0] = X.Sc;
        hd.s[1] = CFG ? X.Su : 0.f;
        hd.s[2] = X.S;
        hd.hs_nP = nP;
        hd.hs_nK = nK;
        hd.hs_nA = nA;
        hd.hs_sep = sk_exact ? 2 : (sep ? 1 : 0);
        hd.hs_sk = s_lo;
        hd.hs_kept = best_kept;
        hd.hs_na = n_above;
        hd.hs_ma = m_above;
        hd.hs_mP = m_bandP;
        hd.hs_nb = n_between;
        hd.hs_mb = m_between;
        hd.handed = 2;
      }
      return true;
    }
  }
  // exact scores of the kept tokens above the bands (they do not depend on
  // the band resolution below)
  Pick bp{kNegInf, kNegInf, 0x7fffffff};
  auto score_tok = [&](int v) {
    const float vals = exact_val<C>(P, X, R, v);
    const float es = exact_score<C>(P, K, v, vals);
    const Pick cand{es, vals, v};
    if (es == es && es > kNegInf && pick_better(cand, bp, K.turbo)) bp = cand;
  };
  for (int q = tid; q < nA && q < C::NT; q += C::NT) score_tok(sm.klist[q]);
  if (nA > C::NT) {
    // more kept tokens than the list holds: all of them, against the best
    // score of the listed ones
    const float thr = red_max1<C>(bp.score, sm, slot);
    kept_pass<C, CFG>(P, X, K, R, S, K2mz, dH, bp, sm, thr);
  }
  // ---- exact resolution of the bands ----
  float Sk = X.S;
  int k_left = 0;
  bool use_k = false;
  if (sep) {
    // S_k: everything above band K plus its first k - n_above members by (exact value, id)
    const int kl = Q.top_k - (int)(n_above + (float)nP + n_between);
    if (kl < 1 || kl > nK) return false;
    float part = 0.f;
    for (int q = tid; q < nK; q += C::NT) {
      const unsigned long long key = sm.cand[C::BAND - 1 - q];
      int rank = 0;
      for (int j2 = 0; j2 < nK; ++j2) rank += (sm.cand[C::BAND - 1 - j2] > key) ? 1 : 0;
      if (rank < kl) part += sm.cande[C::BAND - 1 - q];
    }
    Sk = __fadd_rn(__fadd_rn(__fadd_rn(m_above, m_bandP), fmaxf(m_between, 0.f)), block_sum1<C>(part, sm, slot));
  } else if (topk_on) {
    k_left = Q.top_k - (int)n_above;
    if (k_left < 1 || k_left > nP) return false;
    use_k = true;
  }
  rank_sort<C>(nP, sm);
  if (use_k) {
    float part = 0.f;
    for (int q = tid; q < nP && q < k_left; q += C::NT) part += sm.cande[q];
    Sk = __fadd_rn(m_above, block_sum1<C>(part, sm, slot));
  }
  K.r = __fdiv_rn(1.0f, Sk);
  Band bd;
  bd.n = nP;
  bd.H = 0.f;
  bd.n_above = n_above;
  bd.m_above = m_above;
  bd.overflow = false;
  band_flags<C>(bd, use_k, k_left, topp_on, Q.top_p, K.r, false, 0.f, sm);
  if (topp_on) {
    // the top-p crossing must lie inside band P: its first member kept and,
    // when tokens below the band belong to the top-k set, the band's mass
    // reaching top_p (every token below it then dropped)
    const bool below = sep || !topk_on;
    const bool bad = !sm.cflag[0];
    if (!bad && below && tid < 32) {
      double t = 0.0;
      for (int q = tid; q < nP; q += 32) t += (double)__fmul_rn(sm.cande[q], K.r);
      t = warp_sum_d(t) + (double)m_above * (double)K.r;
      if (tid == 0) sm.hsi[6] = ((float)t >= Q.top_p) ? 0 : 1;
    }
    csync<C>();
    if (bad || (below && sm.hsi[6])) return false;
  }
  // ---- the best kept score: flagged band members and the kept tokens ----
  {
    const Pick b2 = band_pick<C>(P, K, nP, sm);
    if (pick_better(b2, bp, K.turbo)) bp = b2;
  }
  int chosen = block_pick<C>(bp, K.turbo, sm, slot);
  if (chosen < 0) chosen = top1_smem<C>(P, X, R, sm);
  if (tid == 0) {
    if (chosen < 0 || chosen >= V) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      chosen = 0;
    }
    write_choice<C, CFG>(P, R, Q.pos, chosen, X.mc, X.Sc, X.mu, X.Su);
  }
  return true;
}

// One position worked by a group: statistics, group merge, and either the
// whole token choice with the outputs, or (a min-p band of at most 32
// members) the hand-off record for the group's tail warp.
template <class C, bool CFG>
__device__ __forceinline__ void compute_item(const SampleParams& P, KSmem<C>& ks, Smem<C>& sm, int& slot,
                                             int stage, const ItemParams& Q) {
  const int tid = gtid<C>();
  const int V = P.V;
  const int pos = Q.pos;
  const RowRef<C> R = row_ref<C, CFG>(P, ks, stage, pos);
  const float kPosInf = __int_as_float(0x7f800000);
  PosCtx X;
  float sA;
  item_ctx<CFG>(P, Q, X, sA);
  const Span S = make_span<C, CFG>(R, V);
  const bool topk_on = Q.top_k > 0 && Q.top_k < V;
  const bool topp_on = Q.top_p < 1.0f;
  const bool minp_on = Q.min_p > 0.0f;
  const bool band_mode = minp_on && !topk_on;
  const float lg_minp = band_mode ? fminf(log2f(Q.min_p), 0.f) : 0.f;
  Hand& h = ks.hand[stage];
  if (tid == 0) {
    h.n = 0;
    h.handed = 0;
  }
  // top-k / top-p without min-p: the histogram select (three passes)
  if ((topk_on || topp_on) && !minp_on && !(topp_on && !(Q.top_p > 0.0f)))
    if (select_hist<C, CFG>(P, Q, R, S, sm, h)) return;

  // ---- pass 1: this thread's maxima ----
  float mc_t, mu_t, nu_t;
  pass_max<C, CFG>(R, S, mc_t, mu_t, nu_t);
  const float mcr = (mc_t > kNegInf && mc_t < kPosInf) ? mc_t : 0.f;
  const float mur = (mu_t > kNegInf && mu_t < kPosInf) ? mu_t : 0.f;
  // reference for the z2' sum: the bound A2*max(c) - B2*min(u) >= every z2'
  float zr;
  if (X.A2 >= 0.f && X.B2 >= 0.f && mc_t > kNegInf && mc_t < kPosInf &&
      (!CFG || (nu_t > kNegInf && nu_t < kPosInf))) {
    zr = CFG ? __fmaf_rn(mc_t, X.A2, __fmul_rn(-X.B2, nu_t)) : __fmul_rn(mc_t, X.A2);
  } else {
    zr = thread_zmax<C, CFG>(X, R, S);
  }
  if (!(zr > kNegInf)) zr = 0.f;

  // ---- pass 2: sums against the thread references; merged over the group ----
  Stats3 st;
  float vz[C::KV];
  {
    float sc, su, s, dmax;
    pass_sums<C, CFG>(X, R, S, -__fmul_rn(mcr, kLog2e), -__fmul_rn(mur, kLog2e), -zr, sc, su, s, dmax, vz);
    if (s == 0.f && dmax > kNegInf && dmax < kPosInf) {
      // every term underflowed against the bound: use the exact thread maximum
      // (the vector maxima stay relative to the first reference)
      s = pass_resum<C, CFG>(X, R, S, -__fadd_rn(zr, dmax));
      st.ref[2] = __fadd_rn(zr, dmax);
    } else {
      st.ref[2] = zr;
    }
    st.m[0] = mc_t;
    st.ref[0] = __fmul_rn(mcr, kLog2e);
    st.s[0] = sc;
    st.m[1] = CFG ? mu_t : kNegInf;
    st.ref[1] = __fmul_rn(mur, kLog2e);
    st.s[1] = su;
    st.m[2] = dmax > kNegInf ? __fadd_rn(zr, dmax) : kNegInf;
    st.s[2] = s;
  }
  const float mscale[3] = {kLog2e, kLog2e, 1.0f};
  group_merge3<C>(st, mscale, sm, slot);
  stats_core<CFG>(st.m, st.s, X);
  ScoreCtx K;
  bool rest = false;
  auto need_rest = [&]() {
    if (!rest) stats_rest<CFG>(P, Q, sA, X, K);
    rest = true;
  };

  // ---- token choice ----
  int chosen = -1;
  const Pick none{kNegInf, kNegInf, 0x7fffffff};
  if (!(X.Sc == X.Sc) || (CFG && !(X.Su == X.Su))) {
    chosen = 0;  // a NaN/+inf logit makes the whole reference row NaN: argmax -> 0
  } else if (!(X.S == X.S)) {
    const int f = first_nan_or_inf<C>(X, R, V, sm);
    chosen = f < 0 ? 0 : f;
  } else if (!topk_on && !topp_on && !minp_on) {
    // every token kept: server/engine.py:546-550 (or the penalty-only chain)
    need_rest();
    chosen = argmax_smem<C>(P, X, R, -kBig, kBig, 0ull, K, none, sm);
    if (chosen < 0) chosen = 0;
  } else {
    if (band_mode) {
      const float zm = __fadd_rn(X.zmax, lg_minp);
      const float lo_z = __fsub_rn(zm, zmargin(zm));
      // vectors whose largest z2' can reach the band (z2' = z2 - K2 up to rounding)
      uint32_t marks = 0u;
      {
        const float zmp = __fadd_rn(st.m[2], lg_minp);
        const float thr = __fsub_rn(__fsub_rn(__fsub_rn(zmp, zmargin(zmp)),
                                              __fadd_rn(1e-3f, __fmul_rn(4e-6f, __fadd_rn(fabsf(X.K2), fabsf(zmp))))),
                                    zr);  // relative to this thread's reference, as stored
#pragma unroll
        for (int k = 0; k < C::KV; ++k) {
          const bool in_row = S.j0 + tid + k * C::NT < S.j1;
          marks |= (in_row && (vz[k] >= thr || !(thr > kNegInf)) ? 1u : 0u) << k;
        }
      }
      const int n = band_collect<C, CFG>(X, R, S, marks, lo_z, h);
      if (n <= 32 && n > 0) {
        // the group's tail warp resolves it
        if (tid == 0) {
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            h.m[j] = st.m[j];
            h.s[j] = st.s[j];
          }
          h.handed = 1;
        }
        return;
      }
      // a wide band: scored and resolved by the whole group
      need_rest();
      if (tid == 0) sm.misc[0] = 0;
      csync<C>();
      const int n2 = band_marked<C, CFG>(P, X, R, K, S, marks, lo_z, sm);
      if (n2 <= C::BAND && n2 > 0) {
        rank_sort<C>(n2, sm);
        Band bd;
        bd.n = n2;
        bd.H = kBig;
        bd.n_above = 0.f;
        bd.m_above = 0.f;
        bd.overflow = false;
        const float minp_thr = __fmul_rn(Q.min_p, __fmul_rn(sm.cande[0], K.r));
        band_flags<C>(bd, false, 0, topp_on, Q.top_p, K.r, true, minp_thr, sm);
        const Pick bp = band_pick<C>(P, K, bd.n, sm);
        chosen = block_pick<C>(bp, true, sm, slot);
        if (chosen < 0) chosen = cand_id(sm.cand[0]);
      }
    }
    if (chosen < 0) {
      need_rest();
      K.minp_on = minp_on;
      chosen = select_cold<C>(P, X, R, K, Q.top_k, topk_on, topp_on, Q.top_p, Q.min_p, sm);
    }
  }
  if (tid == 0) {
    if (chosen < 0 || chosen >= V) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      chosen = 0;
    }
    write_choice<C, CFG>(P, R, pos, chosen, X.mc, X.Sc, X.mu, X.Su);
  }
}

// One warp resolves a min-p band of n <= 32 members (member `v0` in lane
// < n): exact value, mass and score (penalty + noise) per member, a bitonic
// sort by (exact value, id), top-p / min-p flags from double prefix sums,
// the best kept score, and the outputs.
template <class C, bool CFG>
__device__ __forceinline__ void band_finish_warp(const SampleParams& P, const ItemParams& Q, const PosCtx& X,
                                                 const ScoreCtx& K, int n, int v0, float c0, float u0) {
  const int lane = threadIdx.x & 31;
  const bool live0 = lane < n;
  unsigned long long key = 0ull;
  float e = 0.f, score = kNegInf;
  float cw = c0, uw = u0;  // the logits of the member this lane holds (moved with the sort)
  if (live0) {
    const ScoreIn si = score_in<true>(P, K, v0);
    const float vals = exact_val_cu(P, X, c0, u0);
    key = cand_key(vals, v0);
    e = ex2_approx(__fsub_rn(z2_of(X, c0, u0), X.zmax));
    score = score_from(K, vals, si);
  }
  // bitonic sort, descending key, over the smallest power of two >= n lanes
  int kmax = 2;
  while (kmax < n) kmax <<= 1;
  for (int k = 2; k <= kmax; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, key, j);
      const float ey = __shfl_xor_sync(0xffffffffu, e, j);
      const float sy = __shfl_xor_sync(0xffffffffu, score, j);
      const float cy = __shfl_xor_sync(0xffffffffu, cw, j);
      const float uy = __shfl_xor_sync(0xffffffffu, uw, j);
      const bool up = ((lane & k) == 0) || k == kmax;
      const bool lower = ((lane & j) == 0);
      const bool take_max = (up == lower);
      if (take_max ? (y > key) : (y < key)) {
        key = y;
        e = ey;
        score = sy;
        cw = cy;
        uw = uy;
      }
    }
  }
  const bool live = lane < n;
  const int v = cand_id(key);
  const float p = __fmul_rn(e, K.r);
  double incl = (double)p;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  const float p0 = __shfl_sync(0xffffffffu, p, 0);
  bool keep = live;
  if (Q.top_p < 1.0f) keep = keep && (__fsub_rn((float)incl, p) < Q.top_p);
  keep = keep && (p >= __fmul_rn(Q.min_p, p0));
  float sc = keep ? score : kNegInf;
  if (!(sc == sc)) sc = kNegInf;
  const uint32_t ks2 = sc > kNegInf ? ord_key(sc) : 0u;
  unsigned long long rec = ks2 ? (((unsigned long long)ks2 << 32) | (uint32_t)(31 - lane)) : 0ull;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, rec, o);
    rec = x > rec ? x : rec;
  }
  const int win_lane = rec ? 31 - (int)(uint32_t)(rec & 0xffffffffu) : 0;
  if (lane == win_lane) {
    int chosen = v;
    if (!live || chosen < 0 || chosen >= P.V) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      chosen = 0;
    }
    P.sampled[Q.pos] = chosen;
    if (P.pcu) P.pcu[Q.pos] = pmi_cu<CFG>(X, cw, uw);
  }
  __syncwarp();
}

// Tail warp: the min-p band of the position recorded for `stage`.
template <class C, bool CFG>
__device__ __forceinline__ void tail_finish(const SampleParams& P, KSmem<C>& ks, int stage) {
  const int lane = threadIdx.x & 31;
  const Hand& h = ks.hand[stage];
  const ItemParams Q = h.Q;
  const int n = h.n;
  const RowRef<C> R = row_ref<C, CFG>(P, ks, stage, Q.pos);
  PosCtx X;
  float sA;
  item_ctx<CFG>(P, Q, X, sA);
  float m[3], s[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    m[j] = h.m[j];
    s[j] = h.s[j];
  }
  ScoreCtx K;
  stats_core<CFG>(m, s, X);
  stats_rest<CFG>(P, Q, sA, X, K);
  const int v0 = lane < n ? h.cv[lane] : 0;
  const float c0 = load_elem_smem<C>(R.sc, R.gc, v0);
  const float u0 = CFG ? load_elem_smem<C>(R.su, R.gu, v0) : 0.f;
  band_finish_warp<C, CFG>(P, Q, X, K, n, v0, c0, u0);
}

// Tail warp: the end of a histogram select the group handed over (band K's
// top-k cut and S_k, band P sorted by (exact value, id) with its top-p
// flags, the kept tokens' and kept members' exact scores, the pick and the
// outputs), from the stage's rows, which stay staged until the tail refills
// the stage.  The group handed it over only when its float bounds of S_k
// guarantee the checks below.
template <class C, bool CFG>
__device__ __noinline__ void tail_hist(const SampleParams& P, KSmem<C>& ks, int stage) {
  const int lane = threadIdx.x & 31;
  const Hand& h = ks.hand[stage];
  const ItemParams Q = h.Q;
  const RowRef<C> R = row_ref<C, CFG>(P, ks, stage, Q.pos);
  PosCtx X;
  float sA;
  item_ctx<CFG>(P, Q, X, sA);
  float m[3], s[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    m[j] = h.m[j];
    s[j] = h.s[j];
  }
  ScoreCtx K;
  stats_core<CFG>(m, s, X);
  stats_rest<CFG>(P, Q, sA, X, K);
  const float K2mz = __fsub_rn(X.K2, X.zmax);
  const int nP = h.hs_nP, nK = h.hs_nK, nA = h.hs_nA;
  const float m_above = h.hs_ma;
  auto logits = [&](int v, float& c, float& u) {
    c = load_elem_smem<C>(R.sc, R.gc, v);
    u = CFG ? load_elem_smem<C>(R.su, R.gu, v) : 0.f;
  };
  float Sk = X.S;
  if (h.hs_sep == 2) {
    Sk = h.hs_sk;  // the group computed S_k (band K wider than a warp)
  } else if (h.hs_sep) {
    // S_k: everything above band K plus its first k - n_above members
    const int kl = Q.top_k - (int)(h.hs_na + (float)nP + h.hs_nb);
    unsigned long long key = 0ull;
    float e = 0.f;
    if (lane < nK) {
      const int v = h.kid[lane];
      float c, u;
      logits(v, c, u);
      key = cand_key(exact_val_cu(P, X, c, u), v);
      e = ex2_approx(hdepth<CFG>(X, K2mz, c, u));
    }
    int rank = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) rank += (__shfl_sync(0xffffffffu, key, j) > key) ? 1 : 0;
    const float part = warp_sum(lane < nK && rank < kl ? e : 0.f);
    Sk = __fadd_rn(__fadd_rn(__fadd_rn(m_above, h.hs_mP), fmaxf(h.hs_mb, 0.f)), part);
  }
  // band P: exact values, masses and scores, sorted by (exact value, id)
  const bool live0 = lane < nP;
  unsigned long long key = 0ull;
  float e = 0.f, score = kNegInf;
  if (live0) {
    const int v = h.pid[lane];
    float c, u;
    logits(v, c, u);
    const float vals = exact_val_cu(P, X, c, u);
    key = cand_key(vals, v);
    e = ex2_approx(hdepth<CFG>(X, K2mz, c, u));
    score = exact_score<C>(P, K, v, vals);
  }
  int kmax = 2;
  while (kmax < nP) kmax <<= 1;
  for (int kk = 2; kk <= kmax; kk <<= 1) {
    for (int j = kk >> 1; j > 0; j >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, key, j);
      const float ey = __shfl_xor_sync(0xffffffffu, e, j);
      const float sy = __shfl_xor_sync(0xffffffffu, score, j);
      const bool up = ((lane & kk) == 0) || kk == kmax;
      const bool lower = ((lane & j) == 0);
      if ((up == lower) ? (y > key) : (y < key)) {
        key = y;
        e = ey;
        score = sy;
      }
    }
  }
  const bool live = lane < nP;
  K.r = __fdiv_rn(1.0f, Sk);
  const float p = __fmul_rn(e, K.r);
  double incl = live ? (double)p : 0.0;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  incl += (double)m_above * (double)K.r;
  const bool keep = live && (__fsub_rn((float)incl, p) < Q.top_p);
  // what the group's bounds guaranteed (recorded if the exact values disagree)
  const double tot = __shfl_sync(0xffffffffu, incl, nP - 1);
  if (lane == 0 && (!keep || !((float)tot >= Q.top_p))) atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
  // the best kept score: band P's kept members and the kept tokens above them
  Pick bp{kNegInf, kNegInf, 0x7fffffff};
  if (keep && score == score && score > kNegInf) bp = Pick{score, cand_val(key), cand_id(key)};
  auto consider = [&](int v) {
    float c, u;
    logits(v, c, u);
    const float vals = exact_val_cu(P, X, c, u);
    const float es = exact_score<C>(P, K, v, vals);
    const Pick cand{es, vals, v};
    if (es == es && es > kNegInf && pick_better(cand, bp, K.turbo)) bp = cand;
  };
  if (nA <= 64) {
    for (int i = lane; i < nA; i += 32) consider(h.aid[i]);
  } else if (lane == 0 && h.hs_kept >= 0) {
    consider(h.hs_kept);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Pick y;
    y.score = __shfl_xor_sync(0xffffffffu, bp.score, o);
    y.vals = __shfl_xor_sync(0xffffffffu, bp.vals, o);
    y.v = __shfl_xor_sync(0xffffffffu, bp.v, o);
    if (pick_better(y, bp, K.turbo)) bp = y;
  }
  int chosen = bp.v;
  if (!(bp.score > kNegInf)) {
    // nothing kept scores above -inf: the first sorted candidate (torch's
    // argmax over an all -inf row)
    unsigned long long best = live ? key : 0ull;
    if (nA <= 64) {
      for (int i = lane; i < nA; i += 32) {
        float c, u;
        logits(h.aid[i], c, u);
        const unsigned long long k2 = cand_key(exact_val_cu(P, X, c, u), h.aid[i]);
        best = k2 > best ? k2 : best;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long y = __shfl_xor_sync(0xffffffffu, best, o);
      best = y > best ? y : best;
    }
    chosen = cand_id(best);
  }
  if (lane == 0) {
    if (chosen < 0 || chosen >= P.V) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      chosen = 0;
    }
    P.sampled[Q.pos] = chosen;
    if (P.pcu) {
      float c, u;
      logits(chosen, c, u);
      P.pcu[Q.pos] = pmi_cu<CFG>(X, c, u);
    }
  }
  __syncwarp();
}

// Acquire load of a counter other CTAs update.
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Every CTA of the launch has appended its work-list entries (a bounded
// wait; false if it ran out, and then this CTA claims nothing: the last CTA
// to pass its preamble never waits, so every entry is still claimed).
__device__ __forceinline__ bool preambles_done(const SampleParams& P) {
  if (ld_acquire_u32(P.sched) >= gridDim.x) return true;
  if (P.wait_ns < 0) return false;
  const uint64_t t0 = globaltimer_ns();
  while (ld_acquire_u32(P.sched) < gridDim.x) {
    if (globaltimer_ns() - t0 > (uint64_t)P.wait_ns) return false;
    __nanosleep(200);
  }
  return true;
}

// The parameters of this CTA's local item `it` (one thread).  Static
// schedule: item it is the global entry first + it * stride.  Claimed
// schedule (`dyn`, the select step): items it < n_stat are the CTA's own
// positions (own[]), later ones are claimed from the launch's work list, the
// c-th claim taking entry c, once every CTA has appended its entries.  False:
// no item (every entry claimed, or the other CTAs' entries were not ready in
// time; the CTA then claims nothing more, so that a group's items end at its
// first empty one and no claimed entry is left behind it).
template <class C>
__device__ __forceinline__ bool next_item(const SampleParams& P, KSmem<C>& ks, int it, int n_stat, int first,
                                          int stride, bool dyn, ItemParams& Q) {
  if (!dyn) {
    Q = load_params(P, item_pos<C>(P, first + it * stride));
    return true;
  }
  if (it < n_stat) {
    Q = load_params(P, ks.own[it]);
    return true;
  }
  if (*(volatile int*)&ks.nodyn) return false;
  if (!preambles_done(P)) {
    *(volatile int*)&ks.nodyn = 1;
    return false;
  }
  const int n_list = (int)ld_acquire_u32(P.sched + 1);  // final: every CTA has appended
  const int idx = (int)atomicAdd(P.sched + 2, 1u);
  if (idx >= n_list) return false;
  // another CTA wrote this entry: read it from L2, not from a stale L1 line
  Q = load_params(P, __ldcg(P.work_w + idx));
  return true;
}

// Issue local item Q into `stage`, or (no item) complete the stage's phase
// empty, with Q.pos = -1 for its group.
template <class C>
__device__ __forceinline__ void issue_or_close(const SampleParams& P, KSmem<C>& ks, int stage, bool has,
                                               const ItemParams& Q) {
  if (has) {
    issue_item<C>(P, ks, stage, Q);
  } else {
    ks.hand[stage].Q.pos = -1;
    mbar_arrive_expect_tx(&ks.full[stage], 0u);
  }
  atomicAdd(&ks.issued[stage], 1);
}

// The grouped pipeline over this CTA's items: NG groups of NT threads, each
// working one position at a time from a shared NSTAGE-deep ring of staged
// rows, and one tail warp per group.  Local item `it` uses stage it % NSTAGE
// and group it % NG (NG divides NSTAGE, so each stage serves one group).  The
// group runs the statistics and either finishes the position or hands its
// band to the group's tail warp; the tail warp finishes a handed band, then
// refills a stage its group has released.  Static schedule: n_stat items,
// global entries first + k * stride, the stage of item it refilled with item
// it + NSTAGE.  Claimed schedule (`dyn`): the CTA's own n_stat items, then
// claimed ones; a group stops at its first empty item (claims are made in
// the order of the local items, so every later one is empty too), and when a
// group has two or more stages the refill lags one item (the stage of item
// it - NG takes item it - NG + NSTAGE), so that when the claims run out every
// group holds at most one position besides the one it is working.  Threads
// past C::NTHREADS only take part in the CTA barriers.
template <class C, bool CFG>
__device__ __forceinline__ void group_phase(const SampleParams& P, KSmem<C>& ks, int n_stat, int first, int stride,
                                            bool dyn = false) {
  constexpr int LAG = C::NSTAGE >= 2 * C::NG ? C::NG : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) {
      mbar_init(&ks.full[s], 1);
      mbar_init(&ks.ready[s], C::NW);
      ks.issued[s] = 0;
      ks.landed[s] = 0;
    }
    ks.nodyn = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int n_my = dyn ? 0x7fffffff : n_stat;  // static: the loop bound
  if (threadIdx.x == 0) {
    // the stages may have been read through the generic proxy before
    fence_proxy_async_smem();
    bool more = true;
    for (int s = 0; s < C::NSTAGE && s < n_my; ++s) {
      ItemParams Q{};
      more = more && next_item<C>(P, ks, s, n_stat, first, stride, dyn, Q);
      issue_or_close<C>(P, ks, s, more, Q);
    }
  }
  if (threadIdx.x < C::NG * C::NT) {
    // ---- groups ----
    const int g = gidx<C>();
    const int tid = gtid<C>();
    Smem<C>& sm = ks.g[g];
    int slot = 0;
    for (int it = g; it < n_my; it += C::NG) {
      const int stage = it % C::NSTAGE;
      const uint32_t parity = (uint32_t)(it / C::NSTAGE) & 1u;
      const bool ok = mbar_wait_bounded(&ks.full[stage], parity, P.wait_ns);
      if (!ok) atomicOr(P.status, (unsigned)YAPD_STATUS_WAIT_TIMEOUT);
      if (csync_or<C>(!ok)) break;
      if (tid == 0) atomicAdd(&ks.landed[stage], 1);
      const ItemParams Q = ks.hand[stage].Q;
      const bool empty = Q.pos < 0;
      if (!empty) compute_item<C, CFG>(P, ks, sm, slot, stage, Q);
      __syncwarp();
      if ((threadIdx.x & 31) == 0) mbar_arrive(&ks.ready[stage]);
      if (empty) break;
    }
  } else if (threadIdx.x < C::NTHREADS) {
    // ---- tail warp of group g ----
    const int g = (threadIdx.x - C::NG * C::NT) >> 5;
    const int lane = threadIdx.x & 31;
    for (int it = g; it < n_my; it += C::NG) {
      const int stage = it % C::NSTAGE;
      const uint32_t parity = (uint32_t)(it / C::NSTAGE) & 1u;
      const int ref_it = dyn ? it - LAG + C::NSTAGE : it + C::NSTAGE;
      ItemParams refill{};
      bool has = false;
      if (!dyn && ref_it < n_my) {
        refill = load_params(P, item_pos<C>(P, first + ref_it * stride));
        has = true;
      }
      if (!mbar_wait_bounded(&ks.ready[stage], parity, P.wait_ns)) {
        if (lane == 0) atomicOr(P.status, (unsigned)YAPD_STATUS_WAIT_TIMEOUT);
        break;
      }
      if (ks.hand[stage].Q.pos < 0) break;  // the group's items ended here
      if (ks.hand[stage].handed == 1) tail_finish<C, CFG>(P, ks, stage);
      else if (ks.hand[stage].handed == 2) tail_hist<C, CFG>(P, ks, stage);
      if (lane == 0 && (dyn ? it >= LAG : ref_it < n_my)) {
        if (dyn) has = next_item<C>(P, ks, ref_it, n_stat, first, stride, true, refill);
        fence_proxy_async_smem();
        issue_or_close<C>(P, ks, ref_it % C::NSTAGE, has, refill);
      }
      __syncwarp();
    }
  }
  // copies issued but never waited for (only after a timeout): give them a
  // bounded chance to land before the CTA moves on
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s)
      for (int q = ks.landed[s]; q < ks.issued[s]; ++q)
        (void)mbar_wait_bounded(&ks.full[s], (uint32_t)q & 1u, kWaitLimitNs);
  }
}

// One CTA per SM (grouped pipeline only): token sampling of independent rows
// (yapd_sample_rows) and the fp32 select step.
template <class C, bool CFG>
__global__ void __launch_bounds__(C::NTHREADS, 1) sample_kernel(const __grid_constant__ SampleParams P) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  KSmem<C>& ks = *reinterpret_cast<KSmem<C>*>(smem_raw);
  const int first = blockIdx.x, stride = gridDim.x;
  if (!P.fused) {
    const int n_items = P.n_identity;
    if (first >= n_items) return;
    group_phase<C, CFG>(P, ks, (n_items - first + stride - 1) / stride, first, stride);
    return;
  }
  // select step: each CTA scans its share of the positions, works its first
  // NSTAGE sampled ones itself and appends the rest to the launch's work
  // list; then every CTA claims list entries until none are left, so that
  // CTAs whose positions were cheap take more of them
  const int n_own = cta_prepare_share(P, ks.own, C::NSTAGE, ks.scan);
  __threadfence();  // this CTA's work-list entries before its count below
  __syncthreads();
  if (threadIdx.x == 0) atomicAdd(P.sched, 1u);
  group_phase<C, CFG>(P, ks, n_own, first, stride, true);
  // this CTA's work is done: the state update may be scheduled
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // the last CTA to finish clears the counters for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(P.sched + 3, 1u) == gridDim.x - 1) {
      atomicExch(P.sched, 0u);
      atomicExch(P.sched + 1, 0u);
      atomicExch(P.sched + 2, 0u);
      atomicExch(P.sched + 3, 0u);
    }
  }
}

// ------------------------------------------------------- warp-per-position path
//
// bf16 select step.  Positions in min-p band mode (min-p on, top-k off) are
// worked by teams of T warps (T = 1 when the CTA has at least 9 positions, up
// to 16 when it has one).  Warp r of a team streams chunks r, r + T, ... of
// the position's cond / uncond rows through its own ring of slots (1-D bulk
// copies issued by its lane 0, one mbarrier per slot) and computes, in one
// pass: the exact row maxima (bf16 max), the three sums of exponentials
// against per-lane references (the maxima of the lane's first vector), and
// the vectors that can reach the min-p band (largest z2' against the warp's
// running maximum), which it copies to its stash.  Lanes merge with shuffles,
// warps through shared memory; the band is collected from the stashes and
// resolved by the team's first warp (band_finish_warp, or band_finish_wide
// for up to BANDW members) while the others move on.  Other filter modes,
// wider bands, non-finite rows and rows whose cond / uncond copies differ in
// alignment are deferred to the grouped pipeline, which the same CTA runs
// afterwards over its deferred items.

struct WCfg {
  static constexpr int NWARP = 16;
  static constexpr int NTHREADS = NWARP * 32;
  static constexpr int CHV = 128;            // 16-byte vectors per chunk and row
  static constexpr int CHB = CHV * 16;       // bytes per chunk and row
  static constexpr int NSLOT = 2;            // ring slots per warp
  static constexpr int TPC = CHV / 32;       // vectors per lane and chunk
  static constexpr int MAXCH = ((YAPD_MAX_V * 2 + 15) / 16 + CHV - 1) / CHV;  // chunks per position
  static constexpr int STASH = 64;           // marked vectors a warp keeps on chip per position
  static constexpr int ICAP = 256;           // item positions on chip per CTA
  static constexpr int IREC = 64;            // full item records on chip per CTA
  static constexpr int BANDW = 128;          // widest band the warp path resolves
};
static_assert(WCfg::MAXCH * WCfg::TPC <= 64, "the marks of a position fit one 64-bit word");
static_assert(WCfg::STASH == 64, "the stash compaction holds two entries per lane");
static_assert((WCfg::BANDW & (WCfg::BANDW - 1)) == 0 && WCfg::BANDW >= 64,
              "the band list doubles as a ring of 64 entries or more (a power of two)");
static_assert(WCfg::NTHREADS >= CfgBF16::NTHREADS, "the grouped pipeline runs inside the warp kernel's CTA");

// Work-list entries of deferred positions carry this bit until the CTA
// compacts them (positions are below 2^30).
constexpr int kDeferBit = 1 << 30;

// A position as the warp path sees it.
struct WItem {
  ItemParams Q;
  RowGeom gc, gu;
  Span S;
  int nvi;  // interior vectors S.j1 - S.j0
  int nch;  // chunks
  bool ok;  // eligible for the warp path
};

struct WStash {
  uint4 c[WCfg::STASH];
  uint4 u[WCfg::STASH];
  int j[WCfg::STASH];    // vector index in the row copy
  float z[WCfg::STASH];  // largest z2' of the vector
};

// Band members of a position (ids and logits), then the wide finisher's
// sorted arrays.
struct WBand {
  int n;
  int id[WCfg::BANDW];
  float c[WCfg::BANDW];
  float u[WCfg::BANDW];
  float w[WCfg::BANDW];
};

// A band wider than 32 of a team's last item, resolved by the whole CTA
// after the warp pass (cta_finish_wide) instead of by the leader alone.
struct WPend {
  int n;     // members (0: nothing pending)
  int area;  // the WBand holding them
  ItemParams Q;
  PosCtx X;
  ScoreCtx K;
};

struct WSmem {
  int scan[32];
  int ndef;
  int nflag;  // items this CTA marked deferred
  WPend pend[WCfg::NWARP];
  uint64_t bar[WCfg::NWARP][WCfg::NSLOT];
  float wstat[WCfg::NWARP][2][6];  // per-warp (m, s) of the statistics, by item parity
  WItem item[WCfg::NWARP];         // the position each warp is working (items past IREC)
  WItem irec[WCfg::IREC];           // the CTA's first IREC items
  int items_pos[WCfg::ICAP];        // positions of the CTA's first ICAP items
  ReqTable req;                     // sampling parameters of the first kReqCap requests
  WStash stash[WCfg::NWARP];
  WBand band[WCfg::NWARP];
  alignas(128) unsigned char ring[WCfg::NWARP][WCfg::NSLOT][2 * WCfg::CHB];
};

// The parameters of this CTA's item k (from shared memory for the first
// ICAP items of requests below kReqCap).
__device__ __forceinline__ ItemParams w_params(const SampleParams& P, const WSmem& ws, int k, int first,
                                               int stride) {
  const int pos = k < WCfg::ICAP ? ws.items_pos[k] : (P.work_w[first + k * stride] & ~kDeferBit);
  const int b = pos / P.L;
  if (b >= kReqCap) return load_params(P, pos);
  ItemParams q;
  q.pos = pos;
  q.T = ws.req.T[b];
  q.top_k = ws.req.top_k[b];
  q.top_p = ws.req.top_p[b];
  q.min_p = ws.req.min_p[b];
  q.rep = ws.req.rep[b];
  return q;
}

template <bool CFG>
__device__ __forceinline__ WItem witem(const SampleParams& P, const ItemParams& Q) {
  using C = CfgBF16;
  WItem I;
  I.Q = Q;
  const int b = Q.pos / P.L, l = Q.pos - b * P.L;
  const int64_t base = (int64_t)b * P.stride_req + (int64_t)l * P.stride_pos;
  I.gc = row_geom<C>(P, base);
  I.gu = CFG ? row_geom<C>(P, base + P.stride_branch) : I.gc;
  RowRef<C> R;
  R.sc = R.su = nullptr;
  R.gc = I.gc;
  R.gu = I.gu;
  I.S = make_span<C, CFG>(R, P.V);
  I.nvi = I.S.j1 - I.S.j0;
  I.nch = (I.nvi + WCfg::CHV - 1) / WCfg::CHV;
  const bool topk_on = Q.top_k > 0 && Q.top_k < P.V;
  I.ok = Q.min_p > 0.0f && !topk_on && (!CFG || I.gc.head == I.gu.head) && I.nch <= WCfg::MAXCH &&
         I.S.nscal <= 32;
  return I;
}

// This CTA's item k (the first IREC from shared memory).
template <bool CFG>
__device__ __forceinline__ WItem w_item(const SampleParams& P, const WSmem& ws, int k, int first, int stride) {
  if (k < WCfg::IREC) return ws.irec[k];
  return witem<CFG>(P, w_params(P, ws, k, first, stride));
}

// Team layout of the CTA: NTEAM teams of T warps; team `team`, rank `r`.
struct WTeam {
  int T, NTEAM, team, r;
};

// Copy cursor of a warp (lane 0): chunks r, r + T, ... of the team's
// eligible items k = team, team + NTEAM, ... in order.
struct WCursor {
  int k;            // CTA-local item index
  int q, nch, nvi;  // next chunk, chunks and interior vectors of item k
  const char* c;    // first interior vector of the cond / uncond copies
  const char* u;
  uint32_t gi;      // chunks issued so far
};

// Issue the warp's next chunk into its slot; false at the end of the stream.
template <bool CFG>
__device__ __forceinline__ bool w_issue(const SampleParams& P, WSmem& ws, int warp, const WTeam& tm, int n_my,
                                        int first, int stride, WCursor& c, bool direct = false) {
  while (c.q >= c.nch) {
    c.k += tm.NTEAM;
    if (c.k >= n_my) {
      c.k = n_my;
      c.q = c.nch = 0;
      return false;
    }
    // (`direct`: before the item records exist)
    const WItem I = direct ? witem<CFG>(P, w_params(P, ws, c.k, first, stride)) : w_item<CFG>(P, ws, c.k, first, stride);
    c.q = tm.r;
    c.nch = I.ok ? I.nch : 0;
    c.nvi = I.nvi;
    c.c = I.gc.src + I.S.j0 * 16;
    c.u = I.gu.src + I.S.j0 * 16;
  }
  const int s = (int)(c.gi % WCfg::NSLOT);
  const int nv = min(WCfg::CHV, c.nvi - c.q * WCfg::CHV);
  const uint32_t bytes = (uint32_t)nv * 16u;
  uint64_t* bar = &ws.bar[warp][s];
  mbar_arrive_expect_tx(bar, CFG ? 2u * bytes : bytes);
  bulk_g2s(ws.ring[warp][s], c.c + c.q * WCfg::CHB, bytes, bar);
  if (CFG) bulk_g2s(ws.ring[warp][s] + WCfg::CHB, c.u + c.q * WCfg::CHB, bytes, bar);
  c.q += tm.T;
  ++c.gi;
  return true;
}

__device__ __forceinline__ uint4 ldg128(const char* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// The lane's sums again from global memory against new references (a lane
// whose maxima lie more than 2^100 from its first vector's references).
template <bool CFG>
__device__ __noinline__ void w_resum(const WItem I, const WTeam tm, int lane, float xsc, float xsu, float nmcL,
                                     float nmuL, float nzr, float A2, float nB2, float& sc, float& su, float& s) {
  float a0 = 0.f, b0 = 0.f, c0 = 0.f;
  for (int q = tm.r; q < I.nch; q += tm.T) {
    const int nv = min(WCfg::CHV, I.nvi - q * WCfg::CHV);
    for (int v = lane; v < nv; v += 32) {
      const int j = I.S.j0 + q * WCfg::CHV + v;
      const uint4 a = ldg128(I.gc.src + j * 16);
      uint4 b = a;
      if (CFG) b = ldg128(I.gu.src + j * 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float c = velem<CfgBF16>(a, i);
        a0 += ex2_approx(__fmaf_rn(c, kLog2e, nmcL));
        if (CFG) {
          const float u = velem<CfgBF16>(b, i);
          b0 += ex2_approx(__fmaf_rn(u, kLog2e, nmuL));
          c0 += ex2_approx(__fmaf_rn(c, A2, __fmaf_rn(u, nB2, nzr)));
        } else {
          c0 += ex2_approx(__fmaf_rn(c, A2, nzr));
        }
      }
    }
  }
  if (tm.r == 0 && lane < I.S.nscal) {
    a0 += ex2_approx(__fmaf_rn(xsc, kLog2e, nmcL));
    if (CFG) {
      b0 += ex2_approx(__fmaf_rn(xsu, kLog2e, nmuL));
      c0 += ex2_approx(__fmaf_rn(xsc, A2, __fmaf_rn(xsu, nB2, nzr)));
    } else {
      c0 += ex2_approx(__fmaf_rn(xsc, A2, nzr));
    }
  }
  sc = a0;
  su = b0;
  s = c0;
}

__device__ __forceinline__ float finite_or0(float x) {
  return (x > kNegInf && x < __int_as_float(0x7f800000)) ? x : 0.f;
}

// Barrier over the warps of a team (named barrier 1 + team; one warp: none).
__device__ __forceinline__ void team_sync(const WTeam& tm) {
  if (tm.T > 1) named_sync(1 + tm.team, tm.T * 32);
  else __syncwarp();
}

// Where a warp finds its share of the band {z2 >= lo_z} after the stream:
// its stash entries and the marked vectors the stash could not take (or,
// when the running margins were too thin, all of its vectors), and the
// scalar element of the lane.
struct BandScan {
  float lo_z;
  int nst;
  unsigned long long ovf;
  bool marks;  // the marks cover the band
  bool has_scalar;
  float xsc, xsu;
  int r, T;
};

// f(id, c, u) for every member (z2 >= lo_z) of the lane's share of the band.
template <bool CFG, class F>
__device__ __forceinline__ void for_band_members(const PosCtx& X, const WItem& I, const WStash& st,
                                                 const BandScan& bs, F&& f) {
  using C = CfgBF16;
  const int lane = threadIdx.x & 31;
  auto vec = [&](int j, const uint4& a, const uint4& b) {
    const int v0 = j * C::W - I.S.head;
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      const float c = velem<C>(a, i);
      const float u = CFG ? velem<C>(b, i) : 0.f;
      if (z2_of(X, c, u) >= bs.lo_z) f(v0 + i, c, u);
    }
  };
  if (bs.marks) {
    for (int i = lane; i < min(bs.nst, WCfg::STASH); i += 32) vec(st.j[i], st.c[i], st.u[i]);
    unsigned long long o = bs.ovf;
    while (o) {
      const int bit = __ffsll((long long)o) - 1;
      o &= o - 1ull;
      const int q = bs.r + bs.T * (bit / WCfg::TPC);
      const int j = I.S.j0 + lane + 32 * (bit % WCfg::TPC) + WCfg::CHV * q;
      const uint4 a = ldg128(I.gc.src + j * 16);
      vec(j, a, CFG ? ldg128(I.gu.src + j * 16) : a);
    }
  } else {
    for (int q = bs.r; q < I.nch; q += bs.T) {
      const int nv = min(WCfg::CHV, I.nvi - q * WCfg::CHV);
      for (int v = lane; v < nv; v += 32) {
        const int j = I.S.j0 + q * WCfg::CHV + v;
        const uint4 a = ldg128(I.gc.src + j * 16);
        vec(j, a, CFG ? ldg128(I.gu.src + j * 16) : a);
      }
    }
  }
  if (bs.has_scalar && z2_of(X, bs.xsc, CFG ? bs.xsu : 0.f) >= bs.lo_z) f(scalar_v(I.S, lane), bs.xsc, bs.xsu);
}

// The same share walked by the whole warp in lockstep: f(m, id, c, u) is
// called by every lane for each element slot, m telling whether the lane's
// element there is a member, so that f may use warp collectives.
template <bool CFG, class F>
__device__ __forceinline__ void for_band_members_sync(const PosCtx& X, const WItem& I, const WStash& st,
                                                      const BandScan& bs, F&& f) {
  using C = CfgBF16;
  const int lane = threadIdx.x & 31;
  auto vec = [&](bool has, int j, const uint4& a, const uint4& b) {
    const int v0 = j * C::W - I.S.head;
#pragma unroll 1
    for (int i = 0; i < C::W; ++i) {
      const float c = velem<C>(a, i);
      const float u = CFG ? velem<C>(b, i) : 0.f;
      f(has && z2_of(X, c, u) >= bs.lo_z, v0 + i, c, u);
    }
  };
  const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
  if (bs.marks) {
    const int ns = min(bs.nst, WCfg::STASH);
    for (int base = 0; base < ns; base += 32) {
      const int i = base + lane;
      const bool has = i < ns;
      vec(has, has ? st.j[i] : 0, has ? st.c[i] : zero4, has ? st.u[i] : zero4);
    }
    unsigned long long o = bs.ovf;
    int rounds = __popcll(o);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) rounds = max(rounds, __shfl_xor_sync(0xffffffffu, rounds, s));
    for (int it = 0; it < rounds; ++it) {
      const bool has = o != 0ull;
      int j = 0;
      uint4 a = zero4, b = zero4;
      if (has) {
        const int bit = __ffsll((long long)o) - 1;
        o &= o - 1ull;
        const int q = bs.r + bs.T * (bit / WCfg::TPC);
        j = I.S.j0 + lane + 32 * (bit % WCfg::TPC) + WCfg::CHV * q;
        a = ldg128(I.gc.src + j * 16);
        b = CFG ? ldg128(I.gu.src + j * 16) : a;
      }
      vec(has, j, a, b);
    }
  } else {
    for (int q = bs.r; q < I.nch; q += bs.T) {
      const int nv = min(WCfg::CHV, I.nvi - q * WCfg::CHV);
      for (int v0 = 0; v0 < nv; v0 += 32) {
        const bool has = v0 + lane < nv;
        const int j = I.S.j0 + q * WCfg::CHV + v0 + lane;
        uint4 a = zero4, b = zero4;
        if (has) {
          a = ldg128(I.gc.src + j * 16);
          b = CFG ? ldg128(I.gu.src + j * 16) : a;
        }
        vec(has, j, a, b);
      }
    }
  }
  f(bs.has_scalar && z2_of(X, bs.xsc, CFG ? bs.xsu : 0.f) >= bs.lo_z, scalar_v(I.S, lane), bs.xsc, bs.xsu);
}

// A kept member's (score key, (exact value, -id) key); score key 0 when the
// score is not a number above -inf.  Out of line: one copy of the Philox
// rounds for the whole wide path.
struct WideCand {
  uint32_t ks;
  unsigned long long kk;
};
template <bool CFG>
__device__ __forceinline__ WideCand wide_score(const SampleParams& P, const PosCtx& X, const ScoreCtx& K, int id,
                                               float c, float u) {
  const float vals = exact_val_cu(P, X, c, u);
  const float sc = score_from(K, vals, score_in<false>(P, K, id));
  WideCand w;
  w.ks = (sc == sc && sc > kNegInf) ? ord_key(sc) : 0u;
  w.kk = cand_key(vals, id);
  return w;
}

// The sample of a min-p band too wide for the list, by one warp over the
// members (for_band_members), given the lane's band mass and its member of
// largest z2 from the collection.  Every token ranked above a member has an
// exact value at least the member's, so it lies in the band too: when the
// band's mass is below top_p (less a margin far above the rounding of either
// side's sums) top-p drops no member, and the sample is the best score
// (penalty + noise) among the members min-p keeps, p >= min_p * p0, ties to
// the larger (exact value, -id) key; with nothing kept (scores not numbers)
// the top member is taken -- what band_finish_warp's sort and prefix sums
// give.  p0 is the p of the member of largest z2 (ties to the lower id), the
// top member by (exact value, -id) but where the two orders differ by a
// rounding, which moves the min-p bound by as much.  Returns false, having
// written nothing, when top-p may cut the band.
template <bool CFG>
__device__ __forceinline__ bool wide_minp_pick(const SampleParams& P, const ItemParams Q, const PosCtx X,
                                            const ScoreCtx K, const WItem I, const WStash& st,
                                            const BandScan scan, WBand& B, float bmass, float tz, int tid,
                                            float tc, float tu) {
  const int lane = threadIdx.x & 31;
  if (Q.top_p < 1.0f && !(__fmul_rn(warp_sum(bmass), K.r) < __fsub_rn(Q.top_p, 1e-3f))) return false;
  float wz = tz;
  int wid = tid;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float yz = __shfl_xor_sync(0xffffffffu, wz, o);
    const int yi = __shfl_xor_sync(0xffffffffu, wid, o);
    if (yz > wz || (yz == wz && yi < wid)) {
      wz = yz;
      wid = yi;
    }
  }
  const int tl = __ffs(__ballot_sync(0xffffffffu, tz == wz && tid == wid)) - 1;
  const float p0 = __fmul_rn(ex2_approx(__fsub_rn(wz, X.zmax)), K.r);
  const float thr = __fmul_rn(Q.min_p, p0);
  uint32_t bs = 0u;
  unsigned long long bk = 0ull;
  float bc = 0.f, bu = 0.f;
  // the kept members go through a ring in B (its list is of no use for a
  // band this wide) and are scored 32 at a time, one per lane
  auto score = [&](int slot) {
    const int id = B.id[slot];
    const float c = B.c[slot], u = B.u[slot];
    const WideCand w = wide_score<CFG>(P, X, K, id, c, u);
    if (w.ks > bs || (w.ks == bs && w.kk > bk)) {
      bs = w.ks;
      bk = w.kk;
      bc = c;
      bu = u;
    }
  };
  int head = 0, tail = 0;  // warp-uniform
  for_band_members_sync<CFG>(X, I, st, scan, [&](bool m, int id, float c, float u) {
    const bool keep = m && __fmul_rn(ex2_approx(__fsub_rn(z2_of(X, c, u), X.zmax)), K.r) >= thr;
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    if (bal == 0u) return;
    if (keep) {
      const int at = (tail + __popc(bal & ((1u << lane) - 1u))) & (WCfg::BANDW - 1);
      B.id[at] = id;
      B.c[at] = c;
      B.u[at] = u;
    }
    tail += __popc(bal);
    if (tail - head >= 32) {
      __syncwarp();
      score((head + lane) & (WCfg::BANDW - 1));
      head += 32;
      __syncwarp();
    }
  });
  __syncwarp();
  if (lane < tail - head) score((head + lane) & (WCfg::BANDW - 1));
  uint32_t ws = bs;
  unsigned long long wk = bk;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t ys = __shfl_xor_sync(0xffffffffu, ws, o);
    const unsigned long long yk = __shfl_xor_sync(0xffffffffu, wk, o);
    if (ys > ws || (ys == ws && yk > wk)) {
      ws = ys;
      wk = yk;
    }
  }
  const bool any = ws != 0u;
  const bool mine = any ? (bs == ws && bk == wk) : (lane == tl);
  const unsigned who = __ballot_sync(0xffffffffu, mine);
  if (who == 0u) {
    if (lane == 0) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      P.sampled[Q.pos] = 0;
    }
  } else if (lane == __ffs(who) - 1) {
    int chosen = any ? cand_id(wk) : wid;
    if (chosen < 0 || chosen >= P.V) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      chosen = 0;
    }
    P.sampled[Q.pos] = chosen;
    if (P.pcu) P.pcu[Q.pos] = any ? pmi_cu<CFG>(X, bc, bu) : pmi_cu<CFG>(X, tc, tu);
  }
  __syncwarp();
  return true;
}

// Leader warp: a band of 32 < n <= BANDW members (four per lane).  Exact
// value, mass and score (penalty + noise) per member, the four of a lane
// computed side by side; each member's rank by (exact value, id) and the
// double sum of the masses ranked above it (exact: at most BANDW floats of
// nearby exponents) give the top-p / min-p flags with the arithmetic of
// band_finish_warp's prefix sums; then the best kept score (ties to the lower
// rank).
template <bool CFG>
__device__ __forceinline__ void band_finish_wide(const SampleParams& P, const ItemParams& Q, const PosCtx& X,
                                                 const ScoreCtx& K, WBand& B, int n) {
  using C = CfgBF16;
  constexpr int PER = WCfg::BANDW / 32;
  const int lane = threadIdx.x & 31;
  unsigned long long key[PER];
  float pm[PER], sc[PER], cw[PER], uw[PER];
  int id[PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    const int i = lane + 32 * t;
    const int ic = i < n ? i : 0;
    id[t] = B.id[ic];
    cw[t] = B.c[ic];
    uw[t] = B.u[ic];
  }
  ScoreIn si[PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) si[t] = score_in<true>(P, K, id[t]);
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    const float vals = exact_val_cu(P, X, cw[t], uw[t]);
    key[t] = cand_key(vals, id[t]);
    pm[t] = __fmul_rn(ex2_approx(__fsub_rn(z2_of(X, cw[t], uw[t]), X.zmax)), K.r);
    sc[t] = score_from(K, vals, si[t]);
    if (!(sc[t] == sc[t])) sc[t] = kNegInf;
  }
  __syncwarp();
  // key (high word in c, low word in u) and mass (w) of every member
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    const int i = lane + 32 * t;
    if (i < n) {
      B.c[i] = __uint_as_float((uint32_t)(key[t] >> 32));
      B.u[i] = __uint_as_float((uint32_t)key[t]);
      B.w[i] = pm[t];
    }
  }
  __syncwarp();
  int rank[PER];
  double above[PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    rank[t] = 0;
    above[t] = 0.0;
  }
  double above2[PER];
#pragma unroll
  for (int t = 0; t < PER; ++t) above2[t] = 0.0;
  int j = 0;
  for (; j + 1 < n; j += 2) {
    const unsigned long long k0 =
        ((unsigned long long)__float_as_uint(B.c[j]) << 32) | __float_as_uint(B.u[j]);
    const unsigned long long k1 =
        ((unsigned long long)__float_as_uint(B.c[j + 1]) << 32) | __float_as_uint(B.u[j + 1]);
    const double p0j = (double)B.w[j], p1j = (double)B.w[j + 1];
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const bool u0 = k0 > key[t], u1 = k1 > key[t];
      rank[t] += (u0 ? 1 : 0) + (u1 ? 1 : 0);
      above[t] += u0 ? p0j : 0.0;
      above2[t] += u1 ? p1j : 0.0;
    }
  }
  if (j < n) {
    const unsigned long long kj =
        ((unsigned long long)__float_as_uint(B.c[j]) << 32) | __float_as_uint(B.u[j]);
    const double pj = (double)B.w[j];
#pragma unroll
    for (int t = 0; t < PER; ++t) {
      const bool up = kj > key[t];
      rank[t] += up ? 1 : 0;
      above[t] += up ? pj : 0.0;
    }
  }
#pragma unroll
  for (int t = 0; t < PER; ++t) above[t] += above2[t];
  // the mass of the member ranked first
  float p0l = 0.f;
  bool h0 = false;
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    if (lane + 32 * t < n && rank[t] == 0) {
      p0l = pm[t];
      h0 = true;
    }
  }
  const unsigned b0 = __ballot_sync(0xffffffffu, h0);
  const float p0 = __shfl_sync(0xffffffffu, p0l, b0 ? __ffs(b0) - 1 : 0);
  unsigned long long best = 0ull;
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    if (lane + 32 * t < n) {
      const double incl = above[t] + (double)pm[t];
      bool keep = true;
      if (Q.top_p < 1.0f) keep = __fsub_rn((float)incl, pm[t]) < Q.top_p;
      keep = keep && (pm[t] >= __fmul_rn(Q.min_p, p0));
      if (keep) {
        const uint32_t ks = sc[t] > kNegInf ? ord_key(sc[t]) : 0u;
        const unsigned long long rec =
            ks ? (((unsigned long long)ks << 32) | (uint32_t)(0x7fffffff - rank[t])) : 0ull;
        best = rec > best ? rec : best;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, best, o);
    best = x > best ? x : best;
  }
  const int win = best ? 0x7fffffff - (int)(uint32_t)(best & 0xffffffffu) : 0;
#pragma unroll
  for (int t = 0; t < PER; ++t) {
    if (lane + 32 * t < n && rank[t] == win) {
      int chosen = id[t];
      if (chosen < 0 || chosen >= P.V) {
        atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
        chosen = 0;
      }
      P.sampled[Q.pos] = chosen;
      if (P.pcu) P.pcu[Q.pos] = pmi_cu<CFG>(X, cw[t], uw[t]);
    }
  }
  __syncwarp();
}

// One position by one warp of its team.  Returns false when the team defers
// the position (the same answer in every warp of the team).  `gcons` counts
// the chunks this warp has consumed; `ok_wait` turns false when a slot wait
// expired (the warp then keeps the team's barriers but reads nothing more).
template <bool CFG>
__device__ __forceinline__ bool w_position(const SampleParams& P, WSmem& ws, const WItem& I, int warp,
                                           const WTeam& tm, int parity, bool last, int n_my, int first,
                                           int stride, uint32_t& gcons, WCursor& cur, bool& ok_wait) {
  using C = CfgBF16;
  const int lane = threadIdx.x & 31;
  const ItemParams Q = I.Q;
  if (tm.r == 0 && lane == 0 && P.history_kind != YAPD_HISTORY_NONE && P.history != nullptr && Q.rep != 1.0f) {
    // the request's history row towards L2 for the finish (whole 16-byte blocks inside the row)
    const int b = Q.pos / P.L;
    const bool bits = P.history_kind == YAPD_HISTORY_BITMAP;
    const uintptr_t h0 = reinterpret_cast<uintptr_t>(P.history) + (uintptr_t)((int64_t)b * P.history_stride * (bits ? 4 : 1));
    const uintptr_t hb = h0 + (bits ? (uintptr_t)((P.V + 31) / 32) * 4u : (uintptr_t)P.V);
    const uintptr_t s0 = (h0 + 15) & ~(uintptr_t)15, e0 = hb & ~(uintptr_t)15;
    if (e0 > s0) prefetch_l2(reinterpret_cast<const void*>(s0), (uint32_t)(e0 - s0));
  }
  const float kPosInf = __int_as_float(0x7f800000);
  const int leader = tm.team * tm.T;
  const int area = tm.T > 1 ? leader + parity : warp;
  WBand& B = ws.band[area];
  WStash& st_ = ws.stash[warp];
  PosCtx X;
  float sA;
  item_ctx<CFG>(P, Q, X, sA);
  const float A2 = X.A2, nB2 = -X.B2;
  const float lg_minp = fminf(log2f(Q.min_p), 0.f);
  // scalar elements (partial vectors at the row ends): rank 0, one per lane
  const bool has_scalar = tm.r == 0 && lane < I.S.nscal;
  float xsc = kNegInf, xsu = kNegInf;
  if (has_scalar) {
    const int v = scalar_v(I.S, lane);
    xsc = load_elem_global<C>(I.gc.row, v);
    if (CFG) xsu = load_elem_global<C>(I.gu.row, v);
  }
  const unsigned long long L2p = f2_pack(kLog2e, kLog2e), A2p = f2_pack(A2, A2), nB2p = f2_pack(nB2, nB2);
  const unsigned long long zero = f2_pack(0.f, 0.f);
  uint32_t cm2 = 0xff80ff80u, um2 = 0xff80ff80u;
  unsigned long long scp = zero, sup = zero, sp = zero;
  unsigned long long nrcp = zero, nrup = zero, nrzp = zero;
  float rc = 0.f, ru = 0.f, rz = 0.f;
  float dm = kNegInf, W = kNegInf, mg_min = kBig;
  unsigned long long ovf = 0ull;  // marked vectors the stash could not take
  int nst = 0;                    // stash entries (warp-uniform)
  bool sfull = false;             // a compaction freed little: the stash stays as it is
  bool first_vec = true;
  for (int q = tm.r; q < I.nch; q += tm.T) {
    // after an expired wait nothing more is read (the chunks still count as
    // issued, so the drain at the end waits for them)
    if (!ok_wait) continue;
    const int s = (int)(gcons % WCfg::NSLOT);
    const uint32_t par = (gcons / WCfg::NSLOT) & 1u;
    const bool ok = mbar_wait_bounded(&ws.bar[warp][s], par, P.wait_ns);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) atomicOr(P.status, (unsigned)YAPD_STATUS_WAIT_TIMEOUT);
      ok_wait = false;
      continue;
    }
    ++gcons;
    const int nv = min(WCfg::CHV, I.nvi - q * WCfg::CHV);
    const unsigned char* slot = ws.ring[warp][s];
    if (first_vec) {
      // references: the maxima of this lane's first vector
      first_vec = false;
      if (lane < nv) {
        const uint4 a = lds128(slot + lane * 16);
        uint4 b = a;
        if (CFG) b = lds128(slot + WCfg::CHB + lane * 16);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
        const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
        const uint32_t ac = bmax2(bmax2(a.x, a.y), bmax2(a.z, a.w));
        rc = __fmul_rn(finite_or0(fmaxf(bf16lo(ac), bf16hi(ac))), kLog2e);
        if (CFG) {
          const uint32_t au = bmax2(bmax2(b.x, b.y), bmax2(b.z, b.w));
          ru = __fmul_rn(finite_or0(fmaxf(bf16lo(au), bf16hi(au))), kLog2e);
        }
        float zm = kNegInf;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const unsigned long long cx = f2_bf16(aw[k]);
          const unsigned long long zx =
              CFG ? f2_fma(cx, A2p, f2_fma(f2_bf16(bw[k]), nB2p, zero)) : f2_fma(cx, A2p, zero);
          float lo, hi;
          f2_unpack(zx, lo, hi);
          zm = fmax3(zm, lo, hi);
        }
        rz = finite_or0(zm);
      }
      nrcp = f2_pack(-rc, -rc);
      nrup = f2_pack(-ru, -ru);
      nrzp = f2_pack(-rz, -rz);
    }
    // one 16-byte vector pair: maxima, the three sums, the vector's largest z2'
    auto vec = [&](int v) -> float {
      const uint4 a = lds128(slot + v * 16);
      uint4 b = a;
      if (CFG) b = lds128(slot + WCfg::CHB + v * 16);
      const uint32_t aw[4] = {a.x, a.y, a.z, a.w};
      const uint32_t bw[4] = {b.x, b.y, b.z, b.w};
      cm2 = bmax2(cm2, bmax2(bmax2(a.x, a.y), bmax2(a.z, a.w)));
      if (CFG) um2 = bmax2(um2, bmax2(bmax2(b.x, b.y), bmax2(b.z, b.w)));
      float m = kNegInf;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const unsigned long long cx = f2_bf16(aw[k]);
        unsigned long long dx;
        float lo, hi;
        if (CFG) {
          const unsigned long long ux = f2_bf16(bw[k]);
          dx = f2_fma(cx, A2p, f2_fma(ux, nB2p, nrzp));
          f2_unpack(f2_fma(ux, L2p, nrup), lo, hi);
          sup = f2_add(sup, f2_pack(ex2_approx(lo), ex2_approx(hi)));
        } else {
          dx = f2_fma(cx, A2p, nrzp);
        }
        f2_unpack(f2_fma(cx, L2p, nrcp), lo, hi);
        scp = f2_add(scp, f2_pack(ex2_approx(lo), ex2_approx(hi)));
        f2_unpack(dx, lo, hi);
        sp = f2_add(sp, f2_pack(ex2_approx(lo), ex2_approx(hi)));
        m = fmax3(m, lo, hi);
      }
      dm = fmaxf(dm, m);
      return m;
    };
    float vzl[WCfg::TPC];
    if (nv == WCfg::CHV) {
      // a full chunk: straight-line code over the lane's four vectors
#pragma unroll
      for (int t = 0; t < WCfg::TPC; ++t) vzl[t] = vec(lane + 32 * t);
    } else {
#pragma unroll
      for (int t = 0; t < WCfg::TPC; ++t) vzl[t] = lane + 32 * t < nv ? vec(lane + 32 * t) : kNegInf;
    }
    // marks: vectors whose largest z2' reaches the running maximum + log2(min_p)
    float cmx = vzl[0];
#pragma unroll
    for (int t = 1; t < WCfg::TPC; ++t) cmx = fmaxf(cmx, vzl[t]);
    W = fmaxf(W, warp_max(__fadd_rn(cmx, rz)));
    const float mg = __fadd_rn(0.02f, __fmul_rn(1e-4f, fabsf(W)));
    mg_min = fminf(mg_min, mg);
    const float thr = __fsub_rn(__fadd_rn(W, lg_minp), mg);
    uint32_t mk = 0u;
#pragma unroll
    for (int t = 0; t < WCfg::TPC; ++t)
      mk |= ((__fadd_rn(vzl[t], rz) >= thr || !(thr > kNegInf)) && lane + 32 * t < nv ? 1u : 0u) << t;
    // marked vectors to the stash (warp-aggregated slots)
    const int cnt = __popc(mk);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const int tot = __shfl_sync(0xffffffffu, incl, 31);
    if (nst + tot > WCfg::STASH && nst > 0 && !sfull) {
      // the running maximum has risen: drop the entries now below it
      const int ns = min(nst, WCfg::STASH);
      uint4 ec[2], eu[2];
      int ej[2];
      float ez[2];
      bool keep[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = lane + 32 * h;
        keep[h] = i < ns && st_.z[i] >= thr;
        if (keep[h]) {
          ec[h] = st_.c[i];
          eu[h] = st_.u[i];
          ej[h] = st_.j[i];
          ez[h] = st_.z[i];
        }
      }
      const unsigned kb0 = __ballot_sync(0xffffffffu, keep[0]);
      const unsigned kb1 = __ballot_sync(0xffffffffu, keep[1]);
      __syncwarp();
      const unsigned lt = (1u << lane) - 1u;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (keep[h]) {
          const int d = h == 0 ? __popc(kb0 & lt) : __popc(kb0) + __popc(kb1 & lt);
          st_.c[d] = ec[h];
          st_.u[d] = eu[h];
          st_.j[d] = ej[h];
          st_.z[d] = ez[h];
        }
      }
      __syncwarp();
      nst = __popc(kb0) + __popc(kb1);  // entries past STASH stay in the overflow marks
      // (a wide band: compacting again would free as little)
      sfull = nst > WCfg::STASH - WCfg::STASH / 4;
    }
    int at = nst + incl - cnt;
    nst += tot;
    while (mk) {
      const int t = __ffs(mk) - 1;
      mk &= mk - 1u;
      const int v = lane + 32 * t;
      if (at < WCfg::STASH) {
        st_.c[at] = lds128(slot + v * 16);
        st_.u[at] = CFG ? lds128(slot + WCfg::CHB + v * 16) : make_uint4(0u, 0u, 0u, 0u);
        st_.j[at] = I.S.j0 + q * WCfg::CHV + v;
        st_.z[at] = __fadd_rn(vzl[t], rz);
      } else {
        ovf |= 1ull << ((q / tm.T) * WCfg::TPC + t);
      }
      ++at;
    }
    __syncwarp();
    if (lane == 0) {
      fence_proxy_async_smem();
      (void)w_issue<CFG>(P, ws, warp, tm, n_my, first, stride, cur);
    }
  }
  // lane statistics (with the scalar elements)
  float sc0, sc1, su0, su1, s0, s1;
  f2_unpack(scp, sc0, sc1);
  f2_unpack(sup, su0, su1);
  f2_unpack(sp, s0, s1);
  float sc = sc0 + sc1, su = su0 + su1, s = s0 + s1;
  float mcl = fmaxf(bf16lo(cm2), bf16hi(cm2));
  float mul = CFG ? fmaxf(bf16lo(um2), bf16hi(um2)) : kNegInf;
  if (has_scalar) {
    mcl = fmaxf(mcl, xsc);
    sc += ex2_approx(__fmaf_rn(xsc, kLog2e, -rc));
    float dz;
    if (CFG) {
      mul = fmaxf(mul, xsu);
      su += ex2_approx(__fmaf_rn(xsu, kLog2e, -ru));
      dz = __fmaf_rn(xsc, A2, __fmaf_rn(xsu, nB2, -rz));
    } else {
      dz = __fmaf_rn(xsc, A2, -rz);
    }
    s += ex2_approx(dz);
    dm = fmaxf(dm, dz);
  }
  // a lane whose maxima lie far from its references (more than 2^100 either
  // way: terms could overflow or flush) sums again
  const float zabs = dm > kNegInf ? __fadd_rn(rz, dm) : kNegInf;
  const bool far =
      (mcl > kNegInf && mcl < kPosInf && fabsf(__fsub_rn(__fmul_rn(mcl, kLog2e), rc)) > 100.f) ||
      (CFG && mul > kNegInf && mul < kPosInf && fabsf(__fsub_rn(__fmul_rn(mul, kLog2e), ru)) > 100.f) ||
      (dm > kNegInf && dm < kPosInf && fabsf(dm) > 100.f);
  if (far && ok_wait) {
    rc = __fmul_rn(finite_or0(mcl), kLog2e);
    ru = CFG ? __fmul_rn(finite_or0(mul), kLog2e) : 0.f;
    rz = finite_or0(zabs);
    w_resum<CFG>(I, tm, lane, xsc, xsu, -rc, -ru, -rz, A2, nB2, sc, su, s);
  }
  // merge: lanes (shuffles), then the team's warps (shared memory)
  float m3[3] = {mcl, CFG ? mul : kNegInf, zabs};
  const float r3[3] = {rc, ru, rz};
  // a warp whose wait expired poisons the team's sum: the team defers the
  // position to the grouped pipeline (its own waits decide there)
  float s3[3] = {sc, su, ok_wait ? s : __int_as_float(0x7fc00000)};
  const float mscale[3] = {kLog2e, kLog2e, 1.0f};
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const float Mw = warp_max(m3[j]);
    float sj = s3[j];
    if (m3[j] > kNegInf && Mw < kPosInf) sj = __fmul_rn(sj, ex2_approx(__fsub_rn(r3[j], __fmul_rn(Mw, mscale[j]))));
    m3[j] = Mw;
    s3[j] = warp_sum(sj);
  }
  if (tm.T > 1) {
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        ws.wstat[warp][parity][j] = m3[j];
        ws.wstat[warp][parity][3 + j] = s3[j];
      }
      if (tm.r == 0) B.n = 0;
    }
    team_sync(tm);
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      const float mq = lane < tm.T ? ws.wstat[leader + lane][parity][j] : kNegInf;
      const float sq = lane < tm.T ? ws.wstat[leader + lane][parity][3 + j] : 0.f;
      float M = mq;
      for (int o = 1; o < tm.T; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
      float f = sq;
      if (mq > kNegInf && M < kPosInf)
        f = __fmul_rn(sq, ex2_approx(__fsub_rn(__fmul_rn(mq, mscale[j]), __fmul_rn(M, mscale[j]))));
      for (int o = 1; o < tm.T; o <<= 1) f += __shfl_xor_sync(0xffffffffu, f, o);
      m3[j] = __shfl_sync(0xffffffffu, M, 0);
      s3[j] = __shfl_sync(0xffffffffu, f, 0);
    }
  } else {
    if (lane == 0) B.n = 0;
    __syncwarp();
  }
  stats_core<CFG>(m3, s3, X);
  // (team-uniform: every warp of the team holds the same statistics)
  if (!(X.Sc == X.Sc) || (CFG && !(X.Su == X.Su)) || !(X.S == X.S) || !(X.zmax > kNegInf)) return false;
  ScoreCtx K;
  stats_rest<CFG>(P, Q, sA, X, K);
  // the band {z2 >= lo_z}: stash, overflowed marks, scalar elements
  const float zm = __fadd_rn(X.zmax, lg_minp);
  const float lo_z = __fsub_rn(zm, zmargin(zm));
  const float zmp = __fadd_rn(m3[2], lg_minp);
  const float need = __fadd_rn(zmargin(zmp), __fadd_rn(1e-3f, __fmul_rn(4e-6f, __fadd_rn(fabsf(X.K2), fabsf(zmp)))));
  const BandScan bs{lo_z, nst, ovf, mg_min >= need, has_scalar, xsc, xsu, tm.r, tm.T};
  // collection; alongside, the lane's band mass 2^(z2 - zmax) and its
  // member of largest z2 (ties to the lower id), which a band too wide for
  // the list needs
  float bmass = 0.f, tz = kNegInf, tc = 0.f, tu = 0.f;
  int tid = 0x7fffffff;
  for_band_members<CFG>(X, I, st_, bs, [&](int id, float c, float u) {
    const int at = atomicAdd(&B.n, 1);
    if (at < WCfg::BANDW) {
      B.id[at] = id;
      B.c[at] = c;
      B.u[at] = u;
    }
    const float z = z2_of(X, c, u);
    bmass += ex2_approx(__fsub_rn(z, X.zmax));
    if (z > tz || (z == tz && id < tid)) {
      tz = z;
      tid = id;
      tc = c;
      tu = u;
    }
  });
  team_sync(tm);
  if (tm.r != 0) return true;  // the team's first warp resolves the band
  const int n = B.n;
  // a band too wide for the list, in a one-warp team: resolved here when
  // top-p cannot cut it
  if (n > WCfg::BANDW && tm.T == 1 && wide_minp_pick<CFG>(P, Q, X, K, I, st_, bs, B, bmass, tz, tid, tc, tu))
    return true;
  if (n <= 0 || n > WCfg::BANDW) return false;
  if (n == 1) {
    // a one-member band: min-p keeps it (p >= min_p * p), so does top-p
    // (nothing above it), and an argmax over one kept member (or over none,
    // when its score is not a number) picks it
    if (lane == 0) {
      int chosen = B.id[0];
      if (chosen < 0 || chosen >= P.V) {
        atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
        chosen = 0;
      }
      P.sampled[Q.pos] = chosen;
      if (P.pcu) P.pcu[Q.pos] = pmi_cu<CFG>(X, B.c[0], B.u[0]);
    }
    __syncwarp();
  } else if (n <= 32) {
    const bool live = lane < n;
    band_finish_warp<C, CFG>(P, Q, X, K, n, live ? B.id[lane] : 0, live ? B.c[lane] : 0.f,
                             live ? B.u[lane] : 0.f);
  } else if (last) {
    // the team has no further item: the CTA resolves the band after the warp pass
    if (lane == 0) {
      WPend& pd = ws.pend[warp];
      pd.area = area;
      pd.Q = Q;
      pd.X = X;
      pd.K = K;
      pd.n = n;
    }
    __syncwarp();
  } else {
    band_finish_wide<CFG>(P, Q, X, K, B, n);
  }
  return true;
}

// Scratch of cta_finish_wide, in the ring (free once the warp pass is over).
struct WEpi {
  unsigned long long key[WCfg::BANDW];
  float pm[WCfg::BANDW];
  float sc[WCfg::BANDW];
  unsigned long long best[WCfg::NWARP];
  float p0;
  int win;
};
static_assert(sizeof(WEpi) <= sizeof(((WSmem*)nullptr)->ring), "the wide-band scratch fits the ring");
static_assert(WCfg::NTHREADS >= 4 * WCfg::BANDW, "four threads per band member");

// The band recorded in ws.pend[w], by every thread of the CTA: exact value,
// mass and score per member (one thread each), rank by (exact value, id) and
// the double sum of the masses ranked above (four threads per member), the
// top-p / min-p flags and the best kept score (ties to the lower rank) -- the
// arithmetic of band_finish_wide.
template <bool CFG>
__device__ __noinline__ void cta_finish_wide(const SampleParams& P, WSmem& ws, int w) {
  const WPend& pd = ws.pend[w];
  const int n = pd.n;
  const WBand& B = ws.band[pd.area];
  WEpi& E = *reinterpret_cast<WEpi*>(&ws.ring[0][0][0]);
  const PosCtx X = pd.X;
  const ScoreCtx K = pd.K;
  const ItemParams Q = pd.Q;
  const int lane = threadIdx.x & 31;
  const int i = threadIdx.x >> 2, sub = threadIdx.x & 3;
  const bool own = sub == 0 && i < n;
  float cw = 0.f, uw = 0.f;
  int id = 0;
  if (own) {
    id = B.id[i];
    cw = B.c[i];
    uw = B.u[i];
    const ScoreIn si = score_in<true>(P, K, id);
    const float vals = exact_val_cu(P, X, cw, uw);
    E.key[i] = cand_key(vals, id);
    E.pm[i] = __fmul_rn(ex2_approx(__fsub_rn(z2_of(X, cw, uw), X.zmax)), K.r);
    float sc = score_from(K, vals, si);
    if (!(sc == sc)) sc = kNegInf;
    E.sc[i] = sc;
  }
  __syncthreads();
  int rk = 0;
  double ab = 0.0;
  if (i < n) {
    const unsigned long long ki = E.key[i];
    for (int j = sub; j < n; j += 4) {
      if (E.key[j] > ki) {
        ++rk;
        ab += (double)E.pm[j];
      }
    }
  }
  rk += __shfl_xor_sync(0xffffffffu, rk, 1);
  rk += __shfl_xor_sync(0xffffffffu, rk, 2);
  ab += __shfl_xor_sync(0xffffffffu, ab, 1);
  ab += __shfl_xor_sync(0xffffffffu, ab, 2);
  if (own && rk == 0) E.p0 = E.pm[i];
  __syncthreads();
  unsigned long long rec = 0ull;
  if (own) {
    const float p = E.pm[i];
    const double incl = ab + (double)p;
    bool keep = true;
    if (Q.top_p < 1.0f) keep = __fsub_rn((float)incl, p) < Q.top_p;
    keep = keep && (p >= __fmul_rn(Q.min_p, E.p0));
    const float sc = E.sc[i];
    const uint32_t ks = keep && sc > kNegInf ? ord_key(sc) : 0u;
    rec = ks ? (((unsigned long long)ks << 32) | (uint32_t)(0x7fffffff - rk)) : 0ull;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long x = __shfl_xor_sync(0xffffffffu, rec, o);
    rec = x > rec ? x : rec;
  }
  if (lane == 0) E.best[threadIdx.x >> 5] = rec;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int q = 0; q < WCfg::NWARP; ++q) b = E.best[q] > b ? E.best[q] : b;
    E.win = b ? 0x7fffffff - (int)(uint32_t)(b & 0xffffffffu) : 0;
  }
  __syncthreads();
  if (own && rk == E.win) {
    int chosen = id;
    if (chosen < 0 || chosen >= P.V) {
      atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
      chosen = 0;
    }
    P.sampled[Q.pos] = chosen;
    if (P.pcu) P.pcu[Q.pos] = pmi_cu<CFG>(X, cw, uw);
  }
  __syncthreads();
}

// bf16 select step: preamble, the warp-per-position pass over this CTA's
// items, then the grouped pipeline over the items it deferred.
template <bool CFG>
__global__ void __launch_bounds__(WCfg::NTHREADS, 1) wsample_kernel(const __grid_constant__ SampleParams P) {
  using C = CfgBF16;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  WSmem& ws = *reinterpret_cast<WSmem*>(smem_raw);
  const int n_items = cta_prepare(P, ws.scan, &ws.req, ws.items_pos, WCfg::ICAP);
  const int first = blockIdx.x, stride = gridDim.x;
  if (first >= n_items) return;
  const int n_my = (n_items - first + stride - 1) / stride;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // teams: the fewer the items, the more warps per item
  WTeam tm;
  tm.NTEAM = WCfg::NWARP;
  while (tm.NTEAM > 1 && (tm.NTEAM >> 1) >= n_my) tm.NTEAM >>= 1;
  tm.T = WCfg::NWARP / tm.NTEAM;
  tm.team = warp / tm.T;
  tm.r = warp % tm.T;
  // first copies of each warp (lane 0, its own barriers), then the records of
  // the first IREC items, one thread each
  WCursor cur;
  cur.k = tm.team - tm.NTEAM;
  cur.q = cur.nch = cur.nvi = 0;
  cur.c = cur.u = nullptr;
  cur.gi = 0;
  if (lane == 0) {
    for (int s = 0; s < WCfg::NSLOT; ++s) mbar_init(&ws.bar[warp][s], 1);
    fence_mbar_init();
    ws.pend[warp].n = 0;
    for (int s = 0; s < WCfg::NSLOT; ++s)
      if (!w_issue<CFG>(P, ws, warp, tm, n_my, first, stride, cur, true)) break;
  }
  for (int k = threadIdx.x; k < min(n_my, WCfg::IREC); k += blockDim.x)
    ws.irec[k] = witem<CFG>(P, w_params(P, ws, k, first, stride));
  if (threadIdx.x == 0) ws.nflag = 0;
  __syncthreads();
  uint32_t gcons = 0;
  bool ok_wait = true;
  int parity = 0;
  for (int k = tm.team; k < n_my; k += tm.NTEAM) {
    const int idx = first + k * stride;
    const WItem* Ip = &ws.irec[k < WCfg::IREC ? k : 0];
    if (k >= WCfg::IREC) {
      if (lane == 0) ws.item[warp] = witem<CFG>(P, w_params(P, ws, k, first, stride));
      __syncwarp();
      Ip = &ws.item[warp];
    }
    bool done = false;
    if (Ip->ok) {
      done = w_position<CFG>(P, ws, *Ip, warp, tm, parity, k + tm.NTEAM >= n_my, n_my, first, stride, gcons,
                             cur, ok_wait);
      parity ^= 1;
    }
    if (!done && tm.r == 0 && lane == 0) {
      P.work_w[idx] = Ip->Q.pos | kDeferBit;
      atomicAdd(&ws.nflag, 1);
    }
    __syncwarp();
  }
  // copies issued but not consumed (only after an expired wait)
  const uint32_t gi = __shfl_sync(0xffffffffu, cur.gi, 0);
  if (lane == 0) {
    for (uint32_t g = gcons; g < gi; ++g)
      (void)mbar_wait_bounded(&ws.bar[warp][g % WCfg::NSLOT], (g / WCfg::NSLOT) & 1u, kWaitLimitNs);
    for (int s = 0; s < WCfg::NSLOT; ++s)
      asm volatile("mbarrier.inval.shared::cta.b64 [%0];" ::"r"(smem_u32(&ws.bar[warp][s])) : "memory");
  }
  __syncthreads();
  // wide bands left for the whole CTA (the ring is free now)
  for (int w = 0; w < WCfg::NWARP; ++w)
    if (ws.pend[w].n > 0) cta_finish_wide<CFG>(P, ws, w);
  if (ws.nflag == 0) {
    // nothing deferred: no grouped pass; the state update may be scheduled
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    return;
  }
  // compact the deferred entries to the front of this CTA's work-list slots
  if (warp == 0) {
    int j = 0;
    for (int k0 = 0; k0 < n_my; k0 += 32) {
      const int k = k0 + lane;
      const int e = k < n_my ? P.work_w[first + k * stride] : 0;
      const bool d = k < n_my && (e & kDeferBit);
      const unsigned bal = __ballot_sync(0xffffffffu, d);
      __syncwarp();
      if (d) P.work_w[first + (j + __popc(bal & ((1u << lane) - 1u))) * stride] = e & ~kDeferBit;
      j += __popc(bal);
      __syncwarp();
    }
    if (lane == 0) ws.ndef = j;
  }
  __syncthreads();
  const int n_def = ws.ndef;
  __syncthreads();
  if (n_def > 0) group_phase<C, CFG>(P, *reinterpret_cast<KSmem<C>*>(smem_raw), n_def, first, stride);
}

// ---------------------------------------------------------------- host side

template <class C>
constexpr size_t smem_bytes() {
  return sizeof(KSmem<C>) + 128;
}
static_assert(smem_bytes<CfgBF16>() <= 227 * 1024 && smem_bytes<CfgF32>() <= 227 * 1024 &&
                  smem_bytes<CfgF32R>() <= 227 * 1024,
              "the grouped pipeline's shared memory fits one SM");

static_assert(sizeof(WSmem) + 128 <= 227 * 1024, "the warp kernel's shared memory fits one SM");
constexpr size_t wsmem_bytes() {
  return (sizeof(WSmem) > sizeof(KSmem<CfgBF16>) ? sizeof(WSmem) : sizeof(KSmem<CfgBF16>)) + 128;
}

struct DevInfo {
  int sms = 0;
  int occ[2][2] = {{0, 0}, {0, 0}};  // [bf16][cfg]
  std::atomic<bool> init{false};
};

template <bool CFG>
static int prepare_wkernel() {
  if (cudaFuncSetAttribute(wsample_kernel<CFG>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsmem_bytes()) !=
      cudaSuccess)
    return YAPD_ERR_LAUNCH;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, wsample_kernel<CFG>, WCfg::NTHREADS, wsmem_bytes()) !=
      cudaSuccess)
    return YAPD_ERR_LAUNCH;
  return occ >= 1 ? YAPD_OK : YAPD_ERR_LAUNCH;
}

// Per-device set-up (kernel attributes, SM count), done once per device under
// a lock; a device reset (cudaDeviceReset) is not detected, so a process that
// resets a device must not call the library on it again.
static DevInfo g_dev[64];
static std::mutex g_init_mu;

template <class C, bool CFG>
static int prepare_kernel(int* occ) {
  if (cudaFuncSetAttribute(sample_kernel<C, CFG>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem_bytes<C>()) != cudaSuccess)
    return YAPD_ERR_LAUNCH;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, sample_kernel<C, CFG>, C::NTHREADS, smem_bytes<C>()) !=
      cudaSuccess)
    return YAPD_ERR_LAUNCH;
  return *occ >= 1 ? YAPD_OK : YAPD_ERR_LAUNCH;
}

static int device_info(DevInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return YAPD_ERR_NO_DEVICE;
  DevInfo& d = g_dev[dev];
  if (!d.init.load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_init_mu);
    if (d.init.load(std::memory_order_relaxed)) {
      *out = &d;
      return YAPD_OK;
    }
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return YAPD_ERR_NO_DEVICE;
    int rc = prepare_kernel<CfgBF16, true>(&d.occ[1][1]);
    if (rc == YAPD_OK) rc = prepare_kernel<CfgBF16, false>(&d.occ[1][0]);
    if (rc == YAPD_OK) rc = prepare_kernel<CfgF32, true>(&d.occ[0][1]);
    if (rc == YAPD_OK) rc = prepare_kernel<CfgF32R, false>(&d.occ[0][0]);
    if (rc == YAPD_OK) rc = prepare_wkernel<true>();
    if (rc == YAPD_OK) rc = prepare_wkernel<false>();
    // the state update runs between two sample kernels: the same shared-memory
    // carveout spares the SMs a reconfiguration at each boundary
    if (rc == YAPD_OK && cudaFuncSetAttribute(unmask_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                              (int)cudaSharedmemCarveoutMaxShared) != cudaSuccess)
      rc = YAPD_ERR_LAUNCH;
    if (rc != YAPD_OK) return rc;
    d.init.store(true, std::memory_order_release);
  }
  *out = &d;
  return YAPD_OK;
}

static int fill_sampling(SampleParams& P, const yapd_sampling& s, const yapd_noise& n, int V) {
  P.temperature = s.temperature;
  P.top_k = s.top_k;
  P.top_p = s.top_p;
  P.min_p = s.min_p;
  P.rep_penalty = s.rep_penalty;
  P.temperature_s = s.temperature_s;
  P.top_k_s = s.top_k_s;
  P.top_p_s = s.top_p_s;
  P.min_p_s = s.min_p_s;
  P.rep_penalty_s = s.rep_penalty_s;
  P.zero_temp_greedy = s.zero_temp_greedy;
  if (s.history_kind != YAPD_HISTORY_NONE && s.history_kind != YAPD_HISTORY_BITMAP &&
      s.history_kind != YAPD_HISTORY_BYTES)
    return YAPD_ERR_BAD_ARG;
  if (s.history_kind != YAPD_HISTORY_NONE && !s.history) return YAPD_ERR_NULL_POINTER;
  // a row must hold every token's bit (word v >> 5) or byte (v)
  if (s.history_kind == YAPD_HISTORY_BITMAP && s.history_stride < (int64_t)((V + 31) / 32)) return YAPD_ERR_BAD_SHAPE;
  if (s.history_kind == YAPD_HISTORY_BYTES && s.history_stride < (int64_t)V) return YAPD_ERR_BAD_SHAPE;
  P.history_kind = s.history_kind;
  P.history = s.history;
  P.history_stride = s.history_stride;
  if (n.kind != YAPD_NOISE_PHILOX && n.kind != YAPD_NOISE_EXPLICIT) return YAPD_ERR_BAD_ARG;
  if (n.kind == YAPD_NOISE_EXPLICIT && !n.gumbel_tok) return YAPD_ERR_NULL_POINTER;
  P.noise_kind = n.kind;
  P.seed = n.seed;
  P.offset = n.offset;
  P.gumbel_tok = n.gumbel_tok;
  P.gt_stride_req = n.gt_stride_req;
  P.gt_stride_pos = n.gt_stride_pos;
  return YAPD_OK;
}

template <class C, bool CFG>
static void launch_one(const SampleParams& P0, int occ, int sms, int max_items, cudaStream_t st) {
  int grid = sms * occ;
  if (grid > max_items) grid = max_items;
  if (grid < 1) grid = 1;
  SampleParams P = P0;
  P.div_grid = divu_make(grid);
  sample_kernel<C, CFG><<<grid, C::NTHREADS, smem_bytes<C>(), st>>>(P);
}

static int launch_sample(const SampleParams& P, int dtype, int max_items, cudaStream_t st) {
  DevInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != YAPD_OK) return rc;
  const bool bf = dtype == YAPD_DTYPE_BF16;
  const bool cfg = P.nb == 2;
  const int occ = d->occ[bf ? 1 : 0][cfg ? 1 : 0];
  // the warp kernel's teams serve min-p positions; without min-p anywhere
  // (a scalar min_p <= 0) every position goes to the grouped pipeline, which
  // then runs on its own, without the warp path's code and deferral
  const bool minp_any = P.min_p != nullptr || P.min_p_s > 0.0f;
  if (bf && P.fused && minp_any) {
    // select step: warp-per-position kernel, one CTA per SM
    SampleParams Pw = P;
    Pw.div_grid = divu_make(d->sms);
    if (cfg) wsample_kernel<true><<<d->sms, WCfg::NTHREADS, wsmem_bytes(), st>>>(Pw);
    else wsample_kernel<false><<<d->sms, WCfg::NTHREADS, wsmem_bytes(), st>>>(Pw);
  } else if (bf) {
    if (cfg) launch_one<CfgBF16, true>(P, occ, d->sms, max_items, st);
    else launch_one<CfgBF16, false>(P, occ, d->sms, max_items, st);
  } else {
    if (cfg) launch_one<CfgF32, true>(P, occ, d->sms, max_items, st);
    else launch_one<CfgF32R, false>(P, occ, d->sms, max_items, st);
  }
  return cudaGetLastError() == cudaSuccess ? YAPD_OK : YAPD_ERR_LAUNCH;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

static size_t select_workspace_bytes(int32_t B, int32_t L) {
  if (B <= 0 || L <= 0) return 256;
  const size_t n = (size_t)B * (size_t)L;
  return 256 + align256(n * sizeof(int32_t)) + align256(n * sizeof(float2));
}

// Every host-side check of a select step, before anything is enqueued
// (`need_workspace`: the caller's workspace must be present and large enough).
static int validate_select(const yapd_select_args* a, bool need_workspace) {
  if (!a) return YAPD_ERR_NULL_POINTER;
  if (a->B <= 0 || a->L <= 0 || a->L > YAPD_MAX_L || a->V <= 0 || a->K <= 0 || (a->nb != 1 && a->nb != 2))
    return YAPD_ERR_BAD_SHAPE;
  if (a->V > YAPD_MAX_V) return YAPD_ERR_V_TOO_LARGE;
  if ((int64_t)a->B * a->L > (1 << 30)) return YAPD_ERR_BAD_SHAPE;
  if (a->logits_dtype != YAPD_DTYPE_F32 && a->logits_dtype != YAPD_DTYPE_BF16) return YAPD_ERR_BAD_DTYPE;
  const yapd_engine_state* eng = a->engine;
  if (eng && (!eng->xt_full || !eng->blk_start || !eng->cache_len || !eng->n_speech || !eng->flags))
    return YAPD_ERR_NULL_POINTER;
  if (eng && (eng->blk_limit < 0 || eng->cache_limit < 0 || eng->xt_stride < eng->blk_limit + a->L))
    return YAPD_ERR_BAD_SHAPE;
  if (!a->logits || (!a->xt && !eng) || !a->k_step || !a->is_commit || !a->log_prior || !a->sched_t || !a->q_t ||
      !a->xt_out || !a->sampled || !a->pmi || !a->n_unmask || !a->n_mask_after || !a->hit_eos ||
      !a->k_step_out || !a->is_commit_out)
    return YAPD_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(a->logits) & 15u) != 0) return YAPD_ERR_MISALIGNED;
  if (a->stride_req < 0 || a->stride_branch < 0 || a->stride_pos < 0) return YAPD_ERR_BAD_SHAPE;
  const int64_t last = (int64_t)(a->B - 1) * a->stride_req + (int64_t)(a->nb - 1) * a->stride_branch +
                       (int64_t)(a->L - 1) * a->stride_pos + a->V;
  if (a->logits_numel < last) return YAPD_ERR_BAD_SHAPE;
  if (need_workspace && (!a->workspace || a->workspace_bytes < select_workspace_bytes(a->B, a->L)))
    return YAPD_ERR_WORKSPACE;
  if (a->noise.kind == YAPD_NOISE_EXPLICIT && a->pos_noise && !a->noise.gumbel_pos) return YAPD_ERR_NULL_POINTER;
  SampleParams scratch{};
  return fill_sampling(scratch, a->sampling, a->noise, a->V);
}


}  // namespace yapd

using namespace yapd;

extern "C" {

int yapd_abi_version(void) { return YAPD_ABI_VERSION; }

const char* yapd_status_string(int code) {
  switch (code) {
    case YAPD_OK: return "ok";
    case YAPD_ERR_NULL_POINTER: return "a required pointer is NULL";
    case YAPD_ERR_BAD_SHAPE: return "invalid shape (B, nb, L, V, K or strides)";
    case YAPD_ERR_BAD_DTYPE: return "unsupported logits dtype (f32 or bf16)";
    case YAPD_ERR_MISALIGNED: return "logits base pointer is not 16-byte aligned";
    case YAPD_ERR_V_TOO_LARGE: return "vocabulary larger than YAPD_MAX_V";
    case YAPD_ERR_WORKSPACE: return "workspace missing or too small";
    case YAPD_ERR_LAUNCH: return "CUDA launch failed";
    case YAPD_ERR_BAD_ARG: return "invalid argument";
    case YAPD_ERR_NO_DEVICE: return "no CUDA device";
    default: return "unknown status";
  }
}

size_t yapd_select_workspace_size(int32_t B, int32_t L) { return select_workspace_bytes(B, L); }

size_t yapd_sample_workspace_size(int32_t R) {
  (void)R;
  return 256;
}

int yapd_clear_status(void* workspace, void* stream) {
  if (!workspace) return YAPD_ERR_NULL_POINTER;
  return cudaMemsetAsync(workspace, 0, sizeof(uint32_t), (cudaStream_t)stream) == cudaSuccess
             ? YAPD_OK
             : YAPD_ERR_LAUNCH;
}

int yapd_read_status(const void* workspace, void* stream, uint32_t* status_out) {
  if (!workspace || !status_out) return YAPD_ERR_NULL_POINTER;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyAsync(status_out, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess)
    return YAPD_ERR_LAUNCH;
  return cudaStreamSynchronize(st) == cudaSuccess ? YAPD_OK : YAPD_ERR_LAUNCH;
}

int yapd_select_step(const yapd_select_args* a, void* stream) {
  int rc = validate_select(a, true);
  if (rc != YAPD_OK) return rc;
  const yapd_engine_state* eng = a->engine;

  SampleParams P{};
  const int es = a->logits_dtype == YAPD_DTYPE_BF16 ? 2 : 4;
  P.logits = static_cast<const char*>(a->logits);
  P.logits_end = P.logits + a->logits_numel * es;
  P.stride_req = a->stride_req;
  P.stride_branch = a->stride_branch;
  P.stride_pos = a->stride_pos;
  P.B = a->B;
  P.nb = a->nb;
  P.L = a->L;
  P.div_L = divu_make(a->L);
  P.V = a->V;
  rc = fill_sampling(P, a->sampling, a->noise, a->V);
  if (rc != YAPD_OK) return rc;
  char* ws = static_cast<char*>(a->workspace);
  const size_t n_pos = (size_t)a->B * a->L;
  P.status = reinterpret_cast<uint32_t*>(ws);
  P.work_w = reinterpret_cast<int32_t*>(ws + 256);
  P.pcu = reinterpret_cast<float2*>(ws + 256 + align256(n_pos * sizeof(int32_t)));
  P.sched = reinterpret_cast<uint32_t*>(ws + 64);

  P.n_identity = 0;
  P.cfg_w = a->cfg_scale;
  P.cfg_1pw = a->cfg_one_plus;
  P.sampled = a->sampled;
  P.pos_count = reinterpret_cast<unsigned long long*>(a->positions_sampled);
  P.wait_ns = a->wait_limit_ns == 0 ? kWaitLimitNs : a->wait_limit_ns;
  P.fused = 1;
  P.dense = a->dense ? 1 : 0;

  UnmaskParams& U = P.U;
  U.xt = a->xt;
  U.k_step = a->k_step;
  U.is_commit = a->is_commit;
  U.sched_t = a->sched_t;
  U.q_t = a->q_t;
  U.sampled = a->sampled;
  U.pcu = P.pcu;
  U.log_prior = a->log_prior;
  U.pmi_lambda = a->pmi_lambda;
  U.cfg_w = a->cfg_scale;
  U.cfg_1pw = a->cfg_one_plus;
  U.nb = a->nb;
  U.pmi = a->pmi;
  U.gumbel_pos = a->noise.gumbel_pos;
  U.noise_kind = a->noise.kind;
  U.seed = a->noise.seed;
  U.offset = a->noise.offset;
  U.B = a->B;
  U.L = a->L;
  U.K = a->K;
  U.mask_id = a->mask_id;
  U.stop_id = a->stop_id;
  U.pos_noise = a->pos_noise;
  U.use_quantile = a->use_quantile;
  U.quantile_lerp = a->quantile_lerp ? 1 : 0;
  U.xt_out = a->xt_out;
  U.n_unmask = a->n_unmask;
  U.n_mask_after = a->n_mask_after;
  U.hit_eos = a->hit_eos;
  U.k_step_out = a->k_step_out;
  U.is_commit_out = a->is_commit_out;
  U.xt_full = eng ? eng->xt_full : nullptr;
  U.xt_stride = eng ? eng->xt_stride : 0;
  U.blk_start = eng ? eng->blk_start : nullptr;
  U.cache_len = eng ? eng->cache_len : nullptr;
  U.n_speech = eng ? eng->n_speech : nullptr;
  U.blk_limit = eng ? eng->blk_limit : 0;
  U.cache_limit = eng ? eng->cache_limit : 0;
  U.flags = eng ? eng->flags : nullptr;
  U.status = P.status;

  cudaStream_t st = (cudaStream_t)stream;
  // profiling events: inside a stream capture they must be external event
  // nodes so that graph replays record timestamps
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (a->prof_event_begin || a->prof_event_end) cudaStreamIsCapturing(st, &cap);
  const unsigned ev_flags = cap == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0u;
  if (a->prof_event_begin)
    cudaEventRecordWithFlags(static_cast<cudaEvent_t>(a->prof_event_begin), st, ev_flags);
  // every CTA runs the preamble (work list, output init, idle requests), so
  // the grid is one CTA per SM even when few positions are sampled
  rc = launch_sample(P, a->logits_dtype, 1 << 30, st);
  if (rc != YAPD_OK) return rc;
  if (a->prof_event_end) cudaEventRecordWithFlags(static_cast<cudaEvent_t>(a->prof_event_end), st, ev_flags);
  // the state update may be scheduled while the sampling kernel's last CTAs
  // run; it waits for that kernel's completion on the device
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)((a->B + 3) / 4));
  lc.blockDim = dim3(128);
  lc.dynamicSmemBytes = 0;
  lc.stream = st;
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = la;
  lc.numAttrs = 1;
  if (cudaLaunchKernelEx(&lc, unmask_kernel, U, (int)P.dense) != cudaSuccess) return YAPD_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? YAPD_OK : YAPD_ERR_LAUNCH;
}

int yapd_sample_rows(const yapd_sample_args* a, void* stream) {
  if (!a) return YAPD_ERR_NULL_POINTER;
  if (a->R <= 0 || a->V <= 0) return YAPD_ERR_BAD_SHAPE;
  if (a->V > YAPD_MAX_V) return YAPD_ERR_V_TOO_LARGE;
  if (a->logits_dtype != YAPD_DTYPE_F32 && a->logits_dtype != YAPD_DTYPE_BF16) return YAPD_ERR_BAD_DTYPE;
  if (!a->logits || !a->sampled) return YAPD_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(a->logits) & 15u) != 0) return YAPD_ERR_MISALIGNED;
  if (a->stride_row < 0) return YAPD_ERR_BAD_SHAPE;
  if (a->logits_numel < (int64_t)(a->R - 1) * a->stride_row + a->V) return YAPD_ERR_BAD_SHAPE;
  if (!a->workspace || a->workspace_bytes < yapd_sample_workspace_size(a->R)) return YAPD_ERR_WORKSPACE;
  SampleParams P{};
  const int es = a->logits_dtype == YAPD_DTYPE_BF16 ? 2 : 4;
  P.logits = static_cast<const char*>(a->logits);
  P.logits_end = P.logits + a->logits_numel * es;
  P.stride_req = a->stride_row;
  P.stride_branch = 0;
  P.stride_pos = 0;
  P.B = a->R;
  P.nb = 1;
  P.L = 1;
  P.div_L = divu_make(1);
  P.V = a->V;
  int rc = fill_sampling(P, a->sampling, a->noise, a->V);
  if (rc != YAPD_OK) return rc;
  P.status = static_cast<uint32_t*>(a->workspace);
  P.work_w = nullptr;
  P.fused = 0;
  P.dense = 0;
  P.n_identity = a->R;
  P.sampled = a->sampled;
  P.pcu = nullptr;
  P.wait_ns = a->wait_limit_ns == 0 ? kWaitLimitNs : a->wait_limit_ns;
  return launch_sample(P, a->logits_dtype, a->R, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Select step for callers that cannot allocate device memory.
//
// Some hosts of this library cannot call cudaMalloc at all: a caller running
// inside a memory pool or allocator it does not own, a real-time serving
// loop that forbids allocation after start-up, or a sandbox that only hands
// out pre-registered buffers.  For them, yapd_select_step_noalloc takes its
// scratch (status word, work list and PMI inputs) from one fixed array in
// the library's own device memory instead of a caller workspace.
//
// The array is sized for YAPD_NOALLOC_MAX_POSITIONS positions (B * L); every
// GPU that loads the library holds it until the process exits.  All calls on
// a device share it, and it keeps the previous call's contents: the status
// word is cleared at the start of each call (the rest is fully rewritten
// before it is read), and two calls whose kernels overlap on the GPU (on
// different streams) race on it.
// ---------------------------------------------------------------------------

namespace yapd {

constexpr size_t kNoAllocBytes =
    256 + ((YAPD_NOALLOC_MAX_POSITIONS * sizeof(int32_t) + 255) & ~(size_t)255) +
    ((YAPD_NOALLOC_MAX_POSITIONS * sizeof(float2) + 255) & ~(size_t)255);

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch per device.  In host code the symbol
// name is only a stand-in: the kernels need the address that
// cudaGetSymbolAddress returns with the device current.
static void* g_noalloc_ptr[64];
static std::mutex g_noalloc_mu;

static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return YAPD_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return YAPD_ERR_LAUNCH;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return YAPD_OK;
}

}  // namespace yapd

extern "C" int yapd_select_step_noalloc(const yapd_select_args* args, void* stream) {
  // every argument check first: a rejected call enqueues nothing
  if (!args) return YAPD_ERR_NULL_POINTER;
  if (args->B > 0 && args->L > 0 && (int64_t)args->B * (int64_t)args->L > (int64_t)YAPD_NOALLOC_MAX_POSITIONS)
    return YAPD_ERR_WORKSPACE;
  int rc = validate_select(args, false);
  if (rc != YAPD_OK) return rc;
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != YAPD_OK) return rc;
  if (yapd_select_workspace_size(args->B, args->L) > kNoAllocBytes) return YAPD_ERR_WORKSPACE;
  if (cudaMemsetAsync(scratch, 0, sizeof(uint32_t), (cudaStream_t)stream) != cudaSuccess) return YAPD_ERR_LAUNCH;
  yapd_select_args a = *args;
  a.workspace = scratch;
  a.workspace_bytes = kNoAllocBytes;
  return yapd_select_step(&a, stream);
}

// the fused speech head + select step (tcgen05 GEMM with the select epilogue)
#include "lmhead_select.cuh"
