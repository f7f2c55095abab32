// Fused speech head + select step on the sm_100a tensor cores.
//
// The reference computes the speech logits with a library GEMM
// (server/engine.py:517-520 `speech_head(h)`; inside the CUDA graph,
// chatterbox_flash/engines/flashinfer.py:1452-1461), writes them to HBM and
// then runs the select step over them (server/engine.py:533-558).  Here the
// GEMM logits = hidden . W^T runs on tcgen05 with fp32 accumulators in tensor
// memory, and its epilogue does the select step's per-row work on the
// accumulator tiles as they finish, so logits never reach HBM:
//   - the softmax statistics of the cond and uncond rows (running max and
//     sum of exp, server/engine.py:536-540),
//   - the Gumbel-max scoring (server/engine.py:546-550; with a repetition
//     penalty the filtered chain of server/engine_ar.py:230-243 without
//     top-k / top-p / min-p): every token is scored approximately and the
//     tokens that may still be the argmax are kept as raw (cond, uncond)
//     logit pairs.
// A resolve kernel then merges the statistics and scores the kept tokens
// exactly (the reference's op order), and the unmask kernel finishes the step.
//
// Kept-token rule.  With the final statistics the exact score of token v is
// s(v) = pen(x(v)) + G(v), x(v) = guided/T as the reference rounds it.  The
// epilogue does not know the row's log-sum-exp yet, but x(v) = y(v) + K up to
// rounding, where y(v) = (1+w)/T c_v - w/T u_v and K is the same for every
// token of the position.  With e(v) a bound on that rounding (and on the
// approximate Gumbel transform), the argmax must satisfy
// y + G >= max over unpenalised tokens u of (y(u) + G(u)) - e(v) - e(u):
// the penalty (rep >= 1) only lowers a score.  So each stream keeps every
// token that passes this test against its running maximum, which only
// unpenalised tokens raise.
//
// Data layout.  CTA tile: 128 logit rows x 256 tokens, K in 64-wide blocks
// staged by TMA with the 128-byte swizzle, four stages.  The 128 rows are 64
// positions: each 32-lane group of tensor memory holds 16 positions' cond
// rows (lanes 0-15) and their uncond rows (lanes 16-31), so a thread and its
// partner 16 lanes away hold the two logits of the same token and exchange
// them with one shuffle.  Two accumulator buffers of 256 columns alternate,
// so the MMA of the next tile overlaps the epilogue of this one.  A unit of
// work is (64-position block, one of `parts` token ranges), numbered part by
// part: the CTAs running at one time stream the same weight rows (measured
// faster than numbering block by block, whose parts would share their hidden
// rows in L2 instead: 0.73 against 0.69 ms at B = 512); the resolve kernel
// merges the parts.
#pragma once
#include <cuda.h>  // CUtensorMap and the encode signature (the driver is reached at run time)

namespace yapd {
namespace lm {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_SUB = 32 * BK * 2;       // one 32-row group of the hidden tile: 4 KB
constexpr int A_BYTES = BM * BK * 2;     // 16 KB
constexpr int B_BYTES = BN * BK * 2;     // 32 KB
constexpr int NG = 3;                    // epilogue warps per tensor-memory lane group
constexpr int EPI_WARPS = 4 * NG;
constexpr int NTHREADS = 64 + EPI_WARPS * 32;
constexpr int POS = 64;                  // positions per CTA tile
constexpr int KEEP = 2;                  // kept tokens a thread holds in registers
constexpr int SPILL = 32;                // slots per (position, part) for tokens spilled from full registers
constexpr int FLUSH = 2 * NG * KEEP;     // slots for the registers' survivors: 2 NG threads per (position, part)
constexpr int CAP = SPILL + FLUSH;
constexpr int PARTS_MAX = 8;
constexpr uint32_t TMEM_COLS = 2 * BN;

struct LmParams {
  int B, L, V, D, n_kb, NT, parts, n_mb, n_units, rpc, lh;
  uint32_t idesc_full, idesc_last;
  float2* stats;        // [((p * PARTS_MAX + part) * NG + g) * 2 + branch]: (max, sum exp(x - max)) of warp g
  int32_t* counts;      // [p * PARTS_MAX + part]: 1 + spilled + (flushed << 16); 0 = not published
  int4* cands;          // [(p * PARTS_MAX + part) * CAP + slot]: (v, cond bits, uncond bits, 0); spilled
                        // tokens in slots [0, SPILL), the registers' survivors from SPILL on
  float* dump;          // optional (B, 2, L, V) fp32 logits, for testing
};

struct alignas(1024) LmSmem {
  uint8_t a[STAGES][A_BYTES];
  uint8_t b[STAGES][B_BYTES];
  uint64_t full[STAGES], empty[STAGES], tfull[2], tempty[2], done;
  uint32_t tmem_base;
  int abort_flag;
  int cnt[POS];         // survivors flushed per position
  int spl[POS];         // tokens spilled per position
};

constexpr size_t kSmemBytes = sizeof(LmSmem) + 1024;  // + alignment slack

// ---------------------------------------------------------------- PTX helpers

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] . B[smem]^T, bf16 operands, fp32 accumulate.
__device__ __forceinline__ void umma_bf16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor: K-major tile, rows of 128 bytes with the
// 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;             // leading-dimension offset (unused by swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;   // stride-dimension offset: next 8-row group
  d |= (uint64_t)1u << 46;             // descriptor version of sm_100
  d |= (uint64_t)2u << 61;             // 128-byte swizzle
  return d;
}

// Instruction descriptor of kind::f16: bf16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
      "%7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// 32 consecutive accumulator columns of this thread's lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&x)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 32; ++j) x[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ float lg2_approx(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Gumbel noise of a Philox word, approximately: within 1e-4 of
// gumbel_from_uniform (philox.cuh) on every input.  -ln(u) comes from the
// series -ln(1-e) = e + e^2/2 + e^3/3 (e = 1 - u exact, truncation below
// 3e-7 relative) for u >= 0.99 and from lg2.approx (absolute error below
// 2^-20, i.e. below 1e-4 relative for -ln(u) >= 0.01) otherwise.
__device__ __forceinline__ float gumbel_approx(uint32_t w) {
  const float u = fmaxf(uniform_from_word(w), 1e-20f);
  float E;
  if (u >= 0.99f) {
    const float e = __fsub_rn(1.0f, u);
    E = __fmul_rn(e, __fmaf_rn(e, __fmaf_rn(e, 0.333333333f, 0.5f), 1.0f));
  } else {
    E = __fmul_rn(-lg2_approx(u), kLn2);
  }
  E = fmaxf(E, 1e-20f);
  return __fmul_rn(-lg2_approx(E), kLn2);
}

// Philox4x32-10 (philox.cuh) for the token noise of one position: the
// counter is (q, pos, off_lo, off_hi & 0x7fffffff) with only q varying, so
// the products of the first two rounds that involve the other words are
// computed once per position.
struct PhiloxPos {
  uint32_t k0, k1;          // key
  uint32_t c3;              // counter word 3
  uint32_t r1w0, r1w1;      // round-1 output words 0 and 1 (independent of q)
  uint32_t r2hi0, r2lo0;    // round 2: M0 * (round-1 word 0)
};
constexpr uint32_t kPhM0 = 0xD2511F53u, kPhM1 = 0xCD9E8D57u, kPhW0 = 0x9E3779B9u, kPhW1 = 0xBB67AE85u;

__device__ __forceinline__ PhiloxPos philox_pos(uint64_t seed, uint64_t offset, uint32_t pos) {
  PhiloxPos S;
  S.k0 = (uint32_t)seed;
  S.k1 = (uint32_t)(seed >> 32);
  S.c3 = (uint32_t)(offset >> 32) & 0x7fffffffu;
  const uint32_t c2 = (uint32_t)offset;
  S.r1w0 = __umulhi(kPhM1, c2) ^ pos ^ S.k0;
  S.r1w1 = kPhM1 * c2;
  S.r2hi0 = __umulhi(kPhM0, S.r1w0);
  S.r2lo0 = kPhM0 * S.r1w0;
  return S;
}

// The 4 NB words of counter blocks q0 .. q0+NB-1 (tokens 4*q0 .. 4*(q0+NB)-1),
// the blocks interleaved.
template <int NB>
__device__ __forceinline__ void philox_xn(const PhiloxPos& S, uint32_t q0, uint32_t (&w)[4 * NB]) {
  uint32_t c0[NB], c1[NB], c2[NB], c3[NB];
  uint32_t k0 = S.k0, k1 = S.k1;
#pragma unroll
  for (int i = 0; i < NB; ++i) {  // round 1
    const uint64_t p0 = (uint64_t)kPhM0 * (q0 + (uint32_t)i);  // one wide multiply: both halves
    c0[i] = S.r1w0;
    c1[i] = S.r1w1;
    c2[i] = (uint32_t)(p0 >> 32) ^ S.c3 ^ k1;
    c3[i] = (uint32_t)p0;
  }
  k0 += kPhW0;
  k1 += kPhW1;
#pragma unroll
  for (int i = 0; i < NB; ++i) {  // round 2: word 0 is the same for every block
    const uint64_t p1 = (uint64_t)kPhM1 * c2[i];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1[i] ^ k0, n2 = S.r2hi0 ^ c3[i] ^ k1;
    c0[i] = n0;
    c1[i] = (uint32_t)p1;
    c2[i] = n2;
    c3[i] = S.r2lo0;
  }
#pragma unroll
  for (int r = 2; r < 10; ++r) {
    k0 += kPhW0;
    k1 += kPhW1;
#pragma unroll
    for (int i = 0; i < NB; ++i) {
      const uint64_t p0 = (uint64_t)kPhM0 * c0[i], p1 = (uint64_t)kPhM1 * c2[i];
      const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1[i] ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c3[i] ^ k1;
      c0[i] = n0;
      c1[i] = (uint32_t)p1;
      c2[i] = n2;
      c3[i] = (uint32_t)p0;
    }
  }
#pragma unroll
  for (int i = 0; i < NB; ++i) {
    w[4 * i + 0] = c0[i];
    w[4 * i + 1] = c1[i];
    w[4 * i + 2] = c2[i];
    w[4 * i + 3] = c3[i];
  }
}

__device__ __forceinline__ void lm_abort(LmSmem& sm, uint32_t* status) {
  *reinterpret_cast<volatile int*>(&sm.abort_flag) = 1;
  if (status) atomicOr(status, YAPD_STATUS_WAIT_TIMEOUT);
}
__device__ __forceinline__ bool lm_aborted(LmSmem& sm) {
  return *reinterpret_cast<volatile int*>(&sm.abort_flag) != 0;
}

// Token range [t0, t1) (in 256-wide tiles) of part `part`.
__device__ __forceinline__ void part_tiles(const LmParams& Q, int part, int& t0, int& t1) {
  t0 = part * Q.NT / Q.parts;
  t1 = (part + 1) * Q.NT / Q.parts;
}

// Whether position (b, l) is sampled this step and its request's parameters
// are ones the fused path serves (repetition penalty >= 1; the host checks
// the rest).
__device__ __forceinline__ bool lm_work(const SampleParams& P, int b, int l) {
  const UnmaskParams& U = P.U;
  if (b >= U.B) return false;
  if (!P.dense && (U.is_commit[b] != 0 || xt_at(U, b, l) != U.mask_id)) return false;
  return true;
}
__device__ __forceinline__ bool lm_supported(const SampleParams& P, int b) {
  return param_f(P.rep_penalty, P.rep_penalty_s, b) >= 1.0f;
}

// ---------------------------------------------------------------- roles

// TMA producer (one thread): the hidden tile as four 32-row groups
// (request, 16-position half: cond rows then uncond rows) and the weight tile.
__device__ __forceinline__ void lm_producer(const CUtensorMap* tmA, const CUtensorMap* tmB, const SampleParams& P,
                                            const LmParams& Q, LmSmem& sm) {
  int s = 0;
  uint32_t ph = 0;
  int issued[STAGES];  // parity of the last load issued into each stage, -1: none
#pragma unroll
  for (int i = 0; i < STAGES; ++i) issued[i] = -1;
  bool ok = true;
  for (int u = blockIdx.x; ok && u < Q.n_units; u += gridDim.x) {
    const int part = u / Q.n_mb, mb = u - part * Q.n_mb;
    int t0, t1;
    part_tiles(Q, part, t0, t1);
    for (int t = t0; ok && t < t1; ++t) {
      for (int kb = 0; kb < Q.n_kb; ++kb) {
        if (lm_aborted(sm) || !mbar_wait_bounded(&sm.empty[s], ph ^ 1u, P.wait_ns)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.full[s], A_BYTES + B_BYTES);
        const int k0 = kb * BK;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const int rq = mb * Q.rpc + g / Q.lh, lhi = g % Q.lh;
          tma_load_5d(sm.a[s] + g * A_SUB, tmA, &sm.full[s], k0, 0, lhi, 0, rq);
        }
        tma_load_2d(sm.b[s], tmB, &sm.full[s], k0, t * BN);
        issued[s] = (int)ph;
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
  }
  if (!ok) lm_abort(sm, P.status);
  // no copy may land in shared memory after the CTA has exited
#pragma unroll
  for (int i = 0; i < STAGES; ++i)
    if (issued[i] >= 0) mbar_wait_bounded(&sm.full[i], (uint32_t)issued[i], kWaitLimitNs);
}

// MMA issuer (one thread): per tile, K/16 tcgen05.mma into the accumulator
// buffer the epilogue has released; each stage is released by a commit.
__device__ __forceinline__ void lm_mma(const SampleParams& P, const LmParams& Q, LmSmem& sm, uint32_t tbase) {
  int s = 0, tc = 0;
  uint32_t ph = 0;
  bool ok = true;
  for (int u = blockIdx.x; ok && u < Q.n_units; u += gridDim.x) {
    const int part = u / Q.n_mb;
    int t0, t1;
    part_tiles(Q, part, t0, t1);
    for (int t = t0; ok && t < t1; ++t) {
      const int a = tc & 1;
      const uint32_t aph = (uint32_t)(tc >> 1) & 1u;
      ++tc;
      if (lm_aborted(sm) || !mbar_wait_bounded(&sm.tempty[a], aph ^ 1u, P.wait_ns)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t d = tbase + (uint32_t)(a * BN);
      const uint32_t idesc = t == Q.NT - 1 ? Q.idesc_last : Q.idesc_full;
      for (int kb = 0; kb < Q.n_kb; ++kb) {
        if (lm_aborted(sm) || !mbar_wait_bounded(&sm.full[s], ph, P.wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t da = sw128_desc(smem_u32(sm.a[s])), db = sw128_desc(smem_u32(sm.b[s]));
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)  // +32 bytes of K per step: +2 in the address field
          umma_bf16(d, da + (uint64_t)(2 * k), db + (uint64_t)(2 * k), idesc, (kb | k) != 0 ? 1u : 0u);
        umma_commit(&sm.empty[s]);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (ok) umma_commit(&sm.tfull[a]);
    }
  }
  if (!ok) lm_abort(sm, P.status);
  // every MMA done before tensor memory is released
  umma_commit(&sm.done);
  mbar_wait_bounded(&sm.done, 0u, kWaitLimitNs);
}

struct EpiRow {
  bool act, pen_on, noisy, ovf;
  int b, l, p;
  float A, Bc;               // y = A*c - Bc*u ~ guided/T up to a per-position constant
  float Am, Bg;              // the same as Am * (own row) + Bg * (partner's row)
  const uint32_t* hrow;      // the request's history bitmap row (pen_on)
  float m, S;                // this row's max and sum of exp(x - m) over the columns seen
  float Bh, Mb;              // running max of unpenalised approximate scores, its magnitude
  PhiloxPos ph;              // the position's token-noise generator state
  int kv[KEEP];              // kept tokens (-1: free slot) with their logits,
  float kc[KEEP], ku[KEEP];  // approximate scores and magnitudes
  float ks[KEEP], km[KEEP];
};

// Bound on the rounding of an approximate score against the exact one (up to
// the per-position constant), the Gumbel approximation included, for a token
// and the running maximum together, with a wide safety factor.
__device__ __forceinline__ float keep_margin(const EpiRow& R, float mag, float s) {
  return 2e-3f + 2e-5f * (mag + R.Mb + fabsf(s) + fabsf(R.Bh));
}

// Drop the kept tokens the running maximum has ruled out.
__device__ __forceinline__ void keep_prune(EpiRow& R) {
#pragma unroll
  for (int k = 0; k < KEEP; ++k)
    if (R.kv[k] >= 0 && R.ks[k] < R.Bh - keep_margin(R, R.km[k], R.ks[k])) R.kv[k] = -1;
}

// Into a free register slot; false when every slot holds a token that may still win.
__device__ __forceinline__ bool keep_insert(EpiRow& R, int v, float c, float u, float s, float mag) {
  int at = -1;
#pragma unroll
  for (int k = KEEP - 1; k >= 0; --k)
    if (R.kv[k] < 0) at = k;
  if (at < 0) return false;
#pragma unroll
  for (int k = 0; k < KEEP; ++k)
    if (k == at) {
      R.kv[k] = v;
      R.kc[k] = c;
      R.ku[k] = u;
      R.ks[k] = s;
      R.km[k] = mag;
    }
  return true;
}

// Raise the running maximum to (s, mag) if higher.
__device__ __forceinline__ void keep_raise(EpiRow& R, float s, float mag) {
  if (s > R.Bh) {
    R.Bh = s;
    R.Mb = mag;
    keep_prune(R);
  }
}

// One 32-column chunk of this thread's accumulator row; FULL: all 32 columns
// are tokens (every chunk but the vocabulary's last).
template <bool FULL>
__device__ __forceinline__ void epi_chunk(const SampleParams& P, const LmParams& Q, LmSmem& sm, EpiRow& R,
                                          const float (&x)[32], int v0, uint32_t hw, int part, int pl, int br,
                                          bool dump) {
  const int nval = FULL ? 32 : min(32, Q.V - v0);
  if (dump) {
    float* drow = Q.dump + (((int64_t)R.b * 2 + br) * Q.L + R.l) * Q.V + v0;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nval) drow[j] = x[j];
  }
  // the cond row's value of token j is in the lower half-warp, the uncond
  // row's in the upper: the lower thread scores tokens 0-15 of the chunk,
  // the upper one tokens 16-31
  // mine: this thread's row at its tokens; got: the partner's row there
  float mine[16], got[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    got[j] = __shfl_xor_sync(0xffffffffu, br ? x[j] : x[16 + j], 16);
    mine[j] = br ? x[16 + j] : x[j];
  }
  if (R.act) {
    // statistics of the own row (four independent chains)
    float c4[4] = {kNegInf, kNegInf, kNegInf, kNegInf};
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < nval) c4[j & 3] = fmaxf(c4[j & 3], x[j]);
    const float cm = fmaxf(fmaxf(c4[0], c4[1]), fmaxf(c4[2], c4[3]));
    if (cm > R.m) {
      R.S = __fmul_rn(R.S, ex2_approx(__fmul_rn(__fsub_rn(R.m, cm), kLog2e)));
      R.m = cm;
    }
    const float ml = -__fmul_rn(R.m, kLog2e);
    if (FULL) {  // packed pairs: one f32x2 FMA and one f32x2 add per two elements
      const unsigned long long l2 = f2_pack(kLog2e, kLog2e), m2 = f2_pack(ml, ml);
      unsigned long long acc[2] = {f2_pack(0.f, 0.f), f2_pack(0.f, 0.f)};
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        float e0, e1;
        f2_unpack(f2_fma(f2_pack(x[j], x[j + 1]), l2, m2), e0, e1);
        acc[(j >> 1) & 1] = f2_add(acc[(j >> 1) & 1], f2_pack(ex2_approx(e0), ex2_approx(e1)));
      }
      float s0, s1, s2, s3;
      f2_unpack(acc[0], s0, s1);
      f2_unpack(acc[1], s2, s3);
      R.S = __fadd_rn(R.S, __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3)));
    } else {
      float a4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < nval) a4[j & 3] = __fadd_rn(a4[j & 3], ex2_approx(__fmaf_rn(x[j], kLog2e, ml)));
      R.S = __fadd_rn(R.S, __fadd_rn(__fadd_rn(a4[0], a4[1]), __fadd_rn(a4[2], a4[3])));
    }
    // approximate scores of this thread's 16 tokens, in two halves of 8
    // (shorter live ranges than one pass over 16)
    const bool philox = R.noisy && P.noise_kind != YAPD_NOISE_EXPLICIT;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int vb = v0 + br * 16 + hf * 8;
      const int nv = FULL ? 8 : min(8, Q.V - vb);
      if (nv <= 0) continue;
      const uint32_t hb = (hw >> (vb & 31)) & 0xffu;  // history bits of these tokens
      // approximate scores need no particular rounding (the margins cover
      // it): y = A c - Bc u as Am * mine + Bg * got
      float y[8];
      float ym[2] = {kNegInf, kNegInf}, ma[2] = {0.f, 0.f}, ga[2] = {0.f, 0.f};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        y[j] = __fmaf_rn(R.Am, mine[hf * 8 + j], __fmul_rn(R.Bg, got[hf * 8 + j]));
        if (j < nv) {
          ym[j & 1] = fmaxf(ym[j & 1], y[j]);
          ma[j & 1] = fmaxf(ma[j & 1], fabsf(mine[hf * 8 + j]));
          ga[j & 1] = fmaxf(ga[j & 1], fabsf(got[hf * 8 + j]));
        }
      }
      const float ymax = fmaxf(ym[0], ym[1]);
      // Bound of keep_margin over these tokens: mag <= |A||c| + |Bc||u| <=
      // mgmax, |y| <= mgmax, |G| < 17 for 24-bit uniforms; plus the error of
      // the approximate Gumbel and of the FMA form of y.
      const float mgmax =
          __fmaf_rn(fabsf(R.Am), fmaxf(ma[0], ma[1]), __fmul_rn(fabsf(R.Bg), fmaxf(ga[0], ga[1]))) * 1.0001f;
      const float mb = 2.2e-3f + 2e-5f * (2.0f * mgmax + R.Mb + 17.0f + fabsf(R.Bh));
      uint32_t w[8];
      uint32_t surv = 0u;  // tokens that may pass the keep test
      if (philox) {
        philox_xn<2>(R.ph, (uint32_t)(vb >> 2), w);
        // Gumbel noise obeys G = -ln(-ln u) <= -ln(1 - u) (as -ln u >= 1 - u).
        // A token passes the keep test only if y + G >= Bh - keep_margin,
        // which needs G >= T = Bh - ymax - mb, i.e. 1 - u <= e^-T: every
        // token with a smaller uniform is ruled out by one integer compare.
        uint32_t kthr = 0u;  // in units of the word: uniform u >= k * 2^-24 iff word >= k << 8
        const float T = R.Bh - ymax - mb;
        if (R.Bh > kNegInf && T > 0.0f) {
          const float q = ex2_approx(-T * kLog2e) * 1.0001f;  // e^-T, rounded up past ex2.approx's error
          const float f = (1.0f - q) * 16777216.0f;
          kthr = f > 1.0f ? ((uint32_t)f - 1u) << 8 : 0u;
        }
        uint32_t wmax = 0u;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < nv) wmax = max(wmax, w[j]);
        if (wmax >= kthr) {  // rarely: build the mask
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j < nv && w[j] >= kthr) surv |= 1u << j;
        }
      } else if (R.noisy) {
#pragma unroll
        for (int j = 0; j < 8; ++j) w[j] = 0u;
        surv = (1u << nv) - 1u;  // explicit noise (parity tests): every token
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          w[j] = 0u;
          if (j < nv && y[j] >= R.Bh - mb) surv |= 1u << j;
        }
      }
      while (surv) {
        const int j = __ffs(surv) - 1;
        surv &= surv - 1u;
        float yj = 0.f, mj = 0.f, gj = 0.f;
        uint32_t wj = 0u;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          if (k == j) {
            yj = y[k];
            mj = mine[hf * 8 + k];
            gj = got[hf * 8 + k];
            wj = w[k];
          }
        const float cj = br ? gj : mj, uj = br ? mj : gj;
        const float mgj = __fmaf_rn(fabsf(R.A), fabsf(cj), __fmul_rn(fabsf(R.Bc), fabsf(uj))) * 1.0001f;
        float G = 0.f;
        if (philox)
          G = gumbel_approx(wj);
        else if (R.noisy)
          G = __ldg(P.gumbel_tok + (int64_t)R.b * P.gt_stride_req + (int64_t)R.l * P.gt_stride_pos + vb + j);
        const float sc = R.noisy ? __fadd_rn(yj, G) : yj;
        if (sc >= R.Bh - keep_margin(R, mgj, sc)) {
          if (!((hb >> j) & 1u)) keep_raise(R, sc, mgj);  // penalised tokens never raise it
          if (!keep_insert(R, vb + j, cj, uj, sc, mgj)) {
            // registers full (a cluster of penalised tokens above the running
            // maximum): the token goes to the position's list in memory
            const int slot = atomicAdd(&sm.spl[pl], 1);
            if (slot < SPILL)
              Q.cands[((size_t)R.p * PARTS_MAX + part) * CAP + slot] =
                  make_int4(vb + j, __float_as_int(cj), __float_as_int(uj), 0);
            else
              R.ovf = true;
          }
        }
      }
    }
  }
  // the partner thread scans other tokens of the same position: its running
  // maximum bounds this stream's tokens as well
  const float obh = __shfl_xor_sync(0xffffffffu, R.Bh, 16);
  const float omb = __shfl_xor_sync(0xffffffffu, R.Mb, 16);
  if (R.act) keep_raise(R, obh, omb);
}

// Epilogue warp: drains its lane group's accumulator rows (every NG-th
// 32-column chunk of each tile), then publishes the unit's statistics and
// kept tokens.
__device__ __forceinline__ void lm_epilogue(const SampleParams& P, const LmParams& Q, LmSmem& sm, uint32_t tbase,
                                            int warp, int lane) {
  const int sp = warp & 3;            // the lane group a warp may access is its warp id mod 4
  const int g = (warp - 2) >> 2;      // which of the lane group's NG warps
  const int t16 = lane & 15, br = lane >> 4;
  const int rql = sp / Q.lh, lhi = sp - rql * Q.lh;
  const int pl = sp * 16 + t16;
  const uint32_t lane_addr = tbase + ((uint32_t)(sp * 32) << 16);
  int tc = 0;
  bool bad = false;  // a wait expired: the remaining units only pass the barriers
  for (int u = blockIdx.x; u < Q.n_units; u += gridDim.x) {
    const int part = u / Q.n_mb, mb = u - part * Q.n_mb;
    int t0, t1;
    part_tiles(Q, part, t0, t1);
    EpiRow R;
    R.b = mb * Q.rpc + rql;
    R.l = lhi * 16 + t16;
    R.p = R.b * Q.L + R.l;
    R.act = !bad && lm_work(P, R.b, R.l) && lm_supported(P, R.b);
    R.pen_on = R.noisy = false;
    R.A = R.Bc = R.Am = R.Bg = 0.f;
    R.hrow = nullptr;
    if (R.act) {
      const float T = param_f(P.temperature, P.temperature_s, R.b);
      const float sA = T > 0.0f ? __fdiv_rn(1.0f, T) : 1.0f;
      R.A = __fmul_rn(P.cfg_1pw, sA);
      R.Bc = __fmul_rn(P.cfg_w, sA);
      R.Am = br ? -R.Bc : R.A;
      R.Bg = br ? R.A : -R.Bc;
      const float rep = param_f(P.rep_penalty, P.rep_penalty_s, R.b);
      R.pen_on = P.history_kind == YAPD_HISTORY_BITMAP && P.history != nullptr && rep != 1.0f;
      R.noisy = T > 0.0f || !P.zero_temp_greedy;
      if (R.pen_on) R.hrow = reinterpret_cast<const uint32_t*>(P.history) + (int64_t)R.b * P.history_stride;
      R.ph = philox_pos(P.seed, P.offset, (uint32_t)R.p);
    }
    R.m = kNegInf;
    R.S = 0.f;
    R.Bh = kNegInf;
    R.Mb = 0.f;
    R.ovf = false;
#pragma unroll
    for (int k = 0; k < KEEP; ++k) {
      R.kv[k] = -1;
      R.kc[k] = R.ku[k] = R.ks[k] = R.km[k] = 0.f;
    }
    const bool dump = Q.dump != nullptr && R.b < Q.B && !bad;
    const bool wact = __any_sync(0xffffffffu, R.act || dump);
    for (int t = t0; t < t1; ++t) {
      const int a = tc & 1;
      const uint32_t aph = (uint32_t)(tc >> 1) & 1u;
      // the tile's 32-column chunks c with c = rot (mod NG) are this warp's;
      // the rotation moves with the tile so that the warps share the work
      const int rot = (g + tc) % NG;
      ++tc;
      if (bad) continue;
      const bool arrived = !lm_aborted(sm) && mbar_wait_bounded(&sm.tfull[a], aph, P.wait_ns);
      if (!__all_sync(0xffffffffu, arrived)) {
        bad = true;
        lm_abort(sm, P.status);
        continue;
      }
      tc_fence_after();
      const int ncols = min(BN, Q.V - t * BN);
      const int nct = wact ? (ncols + 31) >> 5 : 0;  // chunks of the tile that hold tokens
      const int nch = nct > rot ? (nct - rot + NG - 1) / NG : 0;
      for (int ch = 0; ch < nch; ++ch) {
        const int c = rot + ch * NG;
        // the chunk's history word, fetched before the accumulator load so
        // that the two latencies overlap
        const uint32_t hw = R.pen_on ? __ldg(R.hrow + ((t * BN + c * 32) >> 5)) : 0u;
        float x[32];
        __syncwarp();
        tmem_ld32(lane_addr + (uint32_t)(a * BN + c * 32), x);
        if (ch == nch - 1) {  // the buffer is free once its last columns are in registers
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.tempty[a]);
        }
        const int v0 = t * BN + c * 32;
        if (v0 + 32 <= Q.V)
          epi_chunk<true>(P, Q, sm, R, x, v0, hw, part, pl, br, dump);
        else
          epi_chunk<false>(P, Q, sm, R, x, v0, hw, part, pl, br, dump);
      }
      if (nch == 0) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sm.tempty[a]);
      }
    }
    if (R.act && !bad) {
      Q.stats[(((size_t)R.p * PARTS_MAX + part) * NG + g) * 2 + br] = make_float2(R.m, R.S);
#pragma unroll
      for (int k = 0; k < KEEP; ++k) {
        if (R.kv[k] < 0) continue;
        const int slot = atomicAdd(&sm.cnt[pl], 1);  // at most FLUSH per position
        Q.cands[((size_t)R.p * PARTS_MAX + part) * CAP + SPILL + slot] =
            make_int4(R.kv[k], __float_as_int(R.kc[k]), __float_as_int(R.ku[k]), 0);
      }
      if (R.ovf) atomicOr(P.status, YAPD_STATUS_CANDIDATE_OVERFLOW);
    }
    named_sync(1, EPI_WARPS * 32);
    if (g == 0 && br == 0) {
      const int nf = sm.cnt[pl], ns = min(sm.spl[pl], SPILL);
      // published only when no role of this CTA failed: the resolve kernel
      // takes a position whose parts are all published
      if (R.act && !lm_aborted(sm)) Q.counts[(size_t)R.p * PARTS_MAX + part] = 1 + ns + (nf << 16);
      sm.cnt[pl] = 0;
      sm.spl[pl] = 0;
    }
    named_sync(1, EPI_WARPS * 32);
  }
}

__global__ void __launch_bounds__(NTHREADS, 1)
    lm_select_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ SampleParams P, const __grid_constant__ LmParams Q) {
  extern __shared__ uint8_t lm_smem_raw[];
  LmSmem& sm = *reinterpret_cast<LmSmem*>((reinterpret_cast<uintptr_t>(lm_smem_raw) + 1023) & ~(uintptr_t)1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
#pragma unroll
    for (int a = 0; a < 2; ++a) {
      mbar_init(&sm.tfull[a], 1);
      mbar_init(&sm.tempty[a], EPI_WARPS);
    }
    mbar_init(&sm.done, 1);
    sm.abort_flag = 0;
    fence_mbar_init();
  }
  if (threadIdx.x < POS) {
    sm.cnt[threadIdx.x] = 0;
    sm.spl[threadIdx.x] = 0;
  }
  if (warp == 1) tmem_alloc(&sm.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = sm.tmem_base;
  if (warp == 0) {
    if (lane == 0) lm_producer(&tmA, &tmB, P, Q, sm);
  } else if (warp == 1) {
    if (lane == 0) lm_mma(P, Q, sm, tbase);
  } else {
    lm_epilogue(P, Q, sm, tbase, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

}  // namespace lm
}  // namespace yapd

namespace yapd {
namespace lm {

// ---------------------------------------------------------------- resolve

struct PickCU {
  Pick k;
  float c, u;
  bool has;
};
__device__ __forceinline__ PickCU pick_merge(const PickCU& a, const PickCU& b, bool turbo) {
  if (!a.has) return b;
  if (!b.has) return a;
  return pick_better(b.k, a.k, turbo) ? b : a;
}

// One warp per position: merge the parts' statistics, score the kept tokens
// exactly (the reference's op order: exact_val_cu, penalize, noise), pick the
// argmax with the reference's tie rule, and write the sampled id and the PMI
// inputs for the unmask kernel.
__device__ __forceinline__ void resolve_position(const SampleParams& P, const LmParams& Q, int p, int b, int l,
                                                 int lane) {
  const size_t base = (size_t)p * PARTS_MAX;
  int cnt = 1;
  if (lane < Q.parts) cnt = Q.counts[base + lane];
  const bool ok = lm_supported(P, b) && __all_sync(0xffffffffu, cnt >= 1);
  if (!ok) {
    if (lane == 0) P.sampled[p] = -2;  // left unsampled: the request is skipped
    return;
  }
  float mc = kNegInf, sc = 0.f, mu = kNegInf, su = 0.f;
  if (lane < NG * Q.parts) {
    const size_t e = ((base + (size_t)(lane / NG)) * NG + (size_t)(lane % NG)) * 2;
    const float2 ec = Q.stats[e], eu = Q.stats[e + 1];
    mc = ec.x;
    sc = ec.y;
    mu = eu.x;
    su = eu.y;
  }
  PosCtx X;
  X.cfg = true;
  X.mc = warp_max(mc);
  X.mu = warp_max(mu);
  const float fc = mc > kNegInf ? __fmul_rn(sc, ex2_approx(__fmul_rn(__fsub_rn(mc, X.mc), kLog2e))) : 0.f;
  const float fu = mu > kNegInf ? __fmul_rn(su, ex2_approx(__fmul_rn(__fsub_rn(mu, X.mu), kLog2e))) : 0.f;
  X.Sc = warp_sum(fc);
  X.Su = warp_sum(fu);
  X.lc = logf(X.Sc);
  X.lu = logf(X.Su);
  X.T = param_f(P.temperature, P.temperature_s, b);
  X.scale = X.T > 0.0f;
  X.rT = X.scale ? __fdiv_rn(1.0f, X.T) : 1.0f;
  ScoreCtx K;
  K.b = b;
  K.pos = p;
  K.l = l;
  K.rep = param_f(P.rep_penalty, P.rep_penalty_s, b);
  K.pen_on = P.history_kind != YAPD_HISTORY_NONE && P.history != nullptr && K.rep != 1.0f;
  K.noisy = X.T > 0.0f || !P.zero_temp_greedy;
  K.turbo = K.pen_on;  // top-k, top-p and min-p are off on this path
  K.minp_on = false;
  K.rrep = K.pen_on ? __fdiv_rn(1.0f, K.rep) : 1.0f;
  K.r = 0.f;
  K.minp_thr = 0.f;
  K.hbits = nullptr;
  PickCU best;
  best.has = false;
  for (int part = 0; part < Q.parts; ++part) {
    const int w = __shfl_sync(0xffffffffu, cnt, part) - 1;
    const int ns = min(w & 0xffff, SPILL), nf = min(w >> 16, FLUSH);
    for (int i = lane; i < ns + nf; i += 32) {
      const int4 e = Q.cands[(base + part) * CAP + (i < ns ? i : SPILL + i - ns)];
      PickCU c;
      c.c = __int_as_float(e.y);
      c.u = __int_as_float(e.z);
      c.k.v = e.x;
      c.k.vals = exact_val_cu(P, X, c.c, c.u);
      c.k.score = score_from(K, c.k.vals, score_in<true>(P, K, e.x));
      c.has = true;
      best = pick_merge(best, c, K.turbo);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    PickCU q;
    q.has = __shfl_xor_sync(0xffffffffu, best.has, o);
    q.k.score = __shfl_xor_sync(0xffffffffu, best.k.score, o);
    q.k.vals = __shfl_xor_sync(0xffffffffu, best.k.vals, o);
    q.k.v = __shfl_xor_sync(0xffffffffu, best.k.v, o);
    q.c = __shfl_xor_sync(0xffffffffu, best.c, o);
    q.u = __shfl_xor_sync(0xffffffffu, best.u, o);
    best = pick_merge(best, q, K.turbo);
  }
  if (lane == 0) {
    if (best.has) {
      P.sampled[p] = best.k.v;
      P.pcu[p] = pmi_cu<true>(X, best.c, best.u);
    } else {
      P.sampled[p] = -2;
      atomicOr(P.status, YAPD_STATUS_INTERNAL);
    }
  }
}

__global__ void __launch_bounds__(256) lm_resolve_kernel(const __grid_constant__ SampleParams P,
                                                         const __grid_constant__ LmParams Q) {
  const int lane = threadIdx.x & 31;
  const int p = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  bool work = false;
  if (p < Q.B * Q.L) {
    const int b = p / Q.L, l = p - b * Q.L;
    work = lm_work(P, b, l);
    if (work) {
      resolve_position(P, Q, p, b, l, lane);
    } else if (lane == 0) {
      P.sampled[p] = -1;
      P.U.pmi[p] = __int_as_float(0x7fc00000);
    }
  }
  const int n = __syncthreads_count(lane == 0 && work);
  if (threadIdx.x == 0 && n > 0 && P.pos_count) atomicAdd(P.pos_count, (unsigned long long)n);
}

}  // namespace lm
}  // namespace yapd

// ---------------------------------------------------------------- host side

namespace yapd {
namespace lm {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's tensor-map encoder, looked up once through the runtime (the
// library does not link the driver library).
static EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

static size_t workspace_bytes(int32_t B, int32_t L) {
  if (B <= 0 || L <= 0) return 256;
  const size_t n = (size_t)B * (size_t)L;
  return 256 + align256(n * sizeof(float2)) + align256(n * PARTS_MAX * sizeof(int32_t)) +
         align256(n * PARTS_MAX * 2 * NG * sizeof(float2)) + align256(n * PARTS_MAX * CAP * sizeof(int4));
}

// Smallest number of token ranges per 64-position block whose units fill the
// SMs' waves to 95 %, else the best filling (at most PARTS_MAX, at most one
// range per tile).
static int choose_parts(int n_mb, int NT, int sms) {
  int best = 1;
  double best_eff = 0.0;
  for (int p = 1; p <= std::min(PARTS_MAX, NT); ++p) {
    const long units = (long)n_mb * p;
    const long waves = (units + sms - 1) / sms;
    const double eff = (double)units / (double)(waves * sms);
    if (eff >= 0.95) return p;
    if (eff > best_eff + 1e-9) {
      best_eff = eff;
      best = p;
    }
  }
  return best;
}

static std::atomic<bool> g_lm_init[64];
static std::mutex g_lm_mu;

static int prepare(int* sms) {
  DevInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != YAPD_OK) return rc;
  *sms = d->sms;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return YAPD_ERR_NO_DEVICE;
  if (!g_lm_init[dev].load(std::memory_order_acquire)) {
    std::lock_guard<std::mutex> lock(g_lm_mu);
    if (!g_lm_init[dev].load(std::memory_order_relaxed)) {
      if (cudaFuncSetAttribute(lm_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) !=
          cudaSuccess)
        return YAPD_ERR_LAUNCH;
      g_lm_init[dev].store(true, std::memory_order_release);
    }
  }
  return encode_fn() ? YAPD_OK : YAPD_ERR_LAUNCH;
}

// Every host-side check of a fused step, before anything is enqueued.
static int validate(const yapd_lmhead_args* h) {
  if (!h) return YAPD_ERR_NULL_POINTER;
  const yapd_select_args* a = &h->select;
  if (a->B <= 0 || a->nb != 2 || (a->L != 16 && a->L != 32) || a->V <= 0 || a->K <= 0) return YAPD_ERR_BAD_SHAPE;
  if (a->V > YAPD_MAX_V) return YAPD_ERR_V_TOO_LARGE;
  if ((int64_t)a->B * a->L > (1 << 28)) return YAPD_ERR_BAD_SHAPE;
  if (h->D < BK || h->D % BK != 0 || h->D > 65536) return YAPD_ERR_BAD_SHAPE;
  if (!h->hidden || !h->weight) return YAPD_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(h->hidden) & 15u) || (reinterpret_cast<uintptr_t>(h->weight) & 15u))
    return YAPD_ERR_MISALIGNED;
  // TMA strides are multiples of 16 bytes (8 bf16 elements)
  if (h->h_stride_req <= 0 || h->h_stride_branch <= 0 || h->h_stride_pos < h->D || (h->h_stride_req % 8) ||
      (h->h_stride_branch % 8) || (h->h_stride_pos % 8) || h->w_stride < h->D || (h->w_stride % 8))
    return YAPD_ERR_BAD_SHAPE;
  const int64_t hlast = (int64_t)(a->B - 1) * h->h_stride_req + h->h_stride_branch +
                        (int64_t)(a->L - 1) * h->h_stride_pos + h->D;
  if (h->hidden_numel < hlast || h->weight_numel < (int64_t)(a->V - 1) * h->w_stride + h->D)
    return YAPD_ERR_BAD_SHAPE;
  const yapd_engine_state* eng = a->engine;
  if (eng && (!eng->xt_full || !eng->blk_start || !eng->cache_len || !eng->n_speech || !eng->flags))
    return YAPD_ERR_NULL_POINTER;
  if (eng && (eng->blk_limit < 0 || eng->cache_limit < 0 || eng->xt_stride < eng->blk_limit + a->L))
    return YAPD_ERR_BAD_SHAPE;
  if ((!a->xt && !eng) || !a->k_step || !a->is_commit || !a->log_prior || !a->sched_t || !a->q_t || !a->xt_out ||
      !a->sampled || !a->pmi || !a->n_unmask || !a->n_mask_after || !a->hit_eos || !a->k_step_out ||
      !a->is_commit_out)
    return YAPD_ERR_NULL_POINTER;
  if (!a->workspace || a->workspace_bytes < workspace_bytes(a->B, a->L)) return YAPD_ERR_WORKSPACE;
  if (a->noise.kind == YAPD_NOISE_EXPLICIT && a->pos_noise && !a->noise.gumbel_pos) return YAPD_ERR_NULL_POINTER;
  // the fused path's sampling chain: no top-k, top-p or min-p, a bitmap history
  const yapd_sampling& s = a->sampling;
  if (s.top_k || s.top_p || s.min_p) return YAPD_ERR_BAD_ARG;
  if ((s.top_k_s > 0 && s.top_k_s < a->V) || !(s.top_p_s >= 1.0f) || s.min_p_s > 0.0f) return YAPD_ERR_BAD_ARG;
  if (s.history_kind == YAPD_HISTORY_BYTES && s.history) return YAPD_ERR_BAD_ARG;
  SampleParams scratch{};
  return fill_sampling(scratch, a->sampling, a->noise, a->V);
}

}  // namespace lm
}  // namespace yapd

extern "C" size_t yapd_lmhead_workspace_size(int32_t B, int32_t L) { return yapd::lm::workspace_bytes(B, L); }

extern "C" int yapd_lmhead_select_step(const yapd_lmhead_args* h, void* stream) {
  using namespace yapd::lm;
  int rc = validate(h);
  if (rc != YAPD_OK) return rc;
  int sms = 0;
  rc = prepare(&sms);
  if (rc != YAPD_OK) return rc;
  const yapd_select_args* a = &h->select;
  const yapd_engine_state* eng = a->engine;

  // tensor maps: hidden as (d, l mod 16, l / 16, branch, request), box
  // (64, 16, 1, 2, 1) = one 32-row group; weight as (d, token), box (64, 256)
  const int lh = a->L / 16;
  CUtensorMap tmA, tmB;
  {
    const cuuint64_t dims[5] = {(cuuint64_t)h->D, 16, (cuuint64_t)lh, 2, (cuuint64_t)a->B};
    const cuuint64_t strides[4] = {(cuuint64_t)h->h_stride_pos * 2, (cuuint64_t)h->h_stride_pos * 32,
                                   (cuuint64_t)h->h_stride_branch * 2, (cuuint64_t)h->h_stride_req * 2};
    const cuuint32_t box[5] = {BK, 16, 1, 2, 1};
    const cuuint32_t es[5] = {1, 1, 1, 1, 1};
    if (encode_fn()(&tmA, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(h->hidden), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return YAPD_ERR_BAD_SHAPE;
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)h->D, (cuuint64_t)a->V};
    const cuuint64_t strides[1] = {(cuuint64_t)h->w_stride * 2};
    const cuuint32_t box[2] = {BK, BN};
    const cuuint32_t es[2] = {1, 1};
    if (encode_fn()(&tmB, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(h->weight), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return YAPD_ERR_BAD_SHAPE;
  }

  SampleParams P{};
  P.B = a->B;
  P.nb = 2;
  P.L = a->L;
  P.div_L = divu_make(a->L);
  P.V = a->V;
  rc = fill_sampling(P, a->sampling, a->noise, a->V);
  if (rc != YAPD_OK) return rc;
  char* ws = static_cast<char*>(a->workspace);
  const size_t n_pos = (size_t)a->B * a->L;
  size_t off = 256;
  P.status = reinterpret_cast<uint32_t*>(ws);
  P.pcu = reinterpret_cast<float2*>(ws + off);
  off += align256(n_pos * sizeof(float2));
  LmParams Q{};
  Q.counts = reinterpret_cast<int32_t*>(ws + off);
  off += align256(n_pos * PARTS_MAX * sizeof(int32_t));
  Q.stats = reinterpret_cast<float2*>(ws + off);
  off += align256(n_pos * PARTS_MAX * 2 * NG * sizeof(float2));
  Q.cands = reinterpret_cast<int4*>(ws + off);
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
  U.nb = 2;
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

  Q.B = a->B;
  Q.L = a->L;
  Q.V = a->V;
  Q.D = h->D;
  Q.n_kb = h->D / BK;
  Q.NT = (a->V + BN - 1) / BN;
  Q.lh = lh;
  Q.rpc = 4 / lh;
  Q.n_mb = (a->B + Q.rpc - 1) / Q.rpc;
  Q.parts = choose_parts(Q.n_mb, Q.NT, sms);
  Q.n_units = Q.n_mb * Q.parts;
  const int last = a->V - (Q.NT - 1) * BN;
  Q.idesc_full = idesc_bf16(BM, BN);
  Q.idesc_last = idesc_bf16(BM, ((last + 15) / 16) * 16);
  Q.dump = h->logits_out;

  cudaStream_t st = (cudaStream_t)stream;
  // nothing is published until this call's GEMM publishes it
  if (cudaMemsetAsync(Q.counts, 0, n_pos * PARTS_MAX * sizeof(int32_t), st) != cudaSuccess) return YAPD_ERR_LAUNCH;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (a->prof_event_begin || a->prof_event_end) cudaStreamIsCapturing(st, &cap);
  const unsigned ev_flags = cap == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0u;
  if (a->prof_event_begin)
    cudaEventRecordWithFlags(static_cast<cudaEvent_t>(a->prof_event_begin), st, ev_flags);
  const int grid = std::min(Q.n_units, sms);
  lm_select_kernel<<<grid, NTHREADS, kSmemBytes, st>>>(tmA, tmB, P, Q);
  if (a->prof_event_end) cudaEventRecordWithFlags(static_cast<cudaEvent_t>(a->prof_event_end), st, ev_flags);
  lm_resolve_kernel<<<(int)((n_pos + 7) / 8), 256, 0, st>>>(P, Q);
  unmask_kernel<<<(a->B + 3) / 4, 128, 0, st>>>(U, P.dense);
  return cudaGetLastError() == cudaSuccess ? YAPD_OK : YAPD_ERR_LAUNCH;
}
