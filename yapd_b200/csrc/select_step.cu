// Block-diffusion select step for B200 (sm_100a).
//
// Kernels (all launched on the caller's stream, no host sync, no allocation):
//   worklist_kernel  compacts the positions that need a token (masked, non-commit)
//   sample_kernel    one persistent CTA per SM slot; each position's cond and
//                    uncond logit rows are staged into shared memory by 1-D bulk
//                    copies (cp.async.bulk + mbarrier, a 3-deep ring) and held in
//                    registers; CFG, temperature, filters, Gumbel-max and PMI are
//                    computed with block reductions (no sort of the vocabulary)
//   unmask_kernel    one warp per request: position noise, quantile threshold,
//                    count schedule, rank, unmask and the state update
//
// Reference semantics: server/engine.py:533-612 and server/engine_ar.py:220-243
// of m8than/yapd (see include/yapd_select.h).  The file is compiled with
// -fmad=false so that every a*b+c the reference rounds twice is rounded twice
// here; contractions that are wanted are written as explicit fmaf.
#include <cuda_runtime.h>
#include <stdint.h>
#include <math.h>

#include "yapd_select.h"
#include "philox.cuh"
#include "select_common.cuh"

namespace yapd {

// ----------------------------------------------------------------- config

template <int NT_, int NVT_, int W_, int ELEM_, int NSTAGE_, int CAP_, int MINB_>
struct KCfg {
  static constexpr int NT = NT_;        // threads per CTA
  static constexpr int NVT = NVT_;      // 16-byte vectors per thread per row
  static constexpr int W = W_;          // elements per 16-byte vector
  static constexpr int ELEM = ELEM_;    // bytes per logit
  static constexpr int NSTAGE = NSTAGE_;
  static constexpr int CAP = CAP_;      // candidate-list capacity (power of two)
  static constexpr int MINB = MINB_;    // CTAs per SM the launch bounds target
  static constexpr int NS = NVT * W;    // element slots per thread per row
  static constexpr int NW = NT / 32;
  static constexpr int ROW_SLOT = ((YAPD_MAX_V * ELEM + 32 + 127) / 128) * 128;
  static constexpr int STAGE_BYTES = 2 * ROW_SLOT;
  static constexpr bool BF16 = (ELEM == 2);
  static_assert(NT * NVT * 16 >= YAPD_MAX_V * ELEM + 32, "row does not fit the thread tile");
};
using CfgBF16 = KCfg<256, 5, 8, 2, 3, 512, 2>;
using CfgF32 = KCfg<512, 5, 4, 4, 3, 1024, 1>;

constexpr uint64_t kWaitLimitNs = 500ull * 1000ull * 1000ull;  // 0.5 s per pipeline wait
constexpr float kMinPMargin = 1e-3f;

// Kernel parameters (flattened from the C ABI structs on the host).
struct SampleParams {
  // logits
  const char* logits;
  const char* logits_end;  // one past the last byte the call may read
  int64_t stride_req, stride_branch, stride_pos;
  int B, nb, L, V;
  // work: positions p = b*L + l; `work` lists them, `work_count` counts them
  const int32_t* work;
  const int32_t* work_count;
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
  // PMI
  const float* log_prior;
  float cfg_w, cfg_1pw, pmi_lambda;
  int want_pmi;
  // outputs
  int32_t* sampled;
  float* pmi;
  uint32_t* status;
};

struct RowGeom {
  const char* src;    // 16-byte aligned copy source
  const char* row;    // element 0 of the row
  uint32_t bytes;     // bulk-copy size (multiple of 16, may be 0)
  int head;           // elements before element 0 in the copy
  int avail;          // elements [0, avail) are inside the copy
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

__device__ __forceinline__ bool history_has(const SampleParams& P, int b, int v) {
  if (P.history_kind == YAPD_HISTORY_BITMAP) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(P.history) + (int64_t)b * P.history_stride;
    return (__ldg(w + (v >> 5)) >> (v & 31)) & 1u;
  }
  if (P.history_kind == YAPD_HISTORY_BYTES) {
    const uint8_t* h = reinterpret_cast<const uint8_t*>(P.history) + (int64_t)b * P.history_stride;
    return __ldg(h + v) != 0;
  }
  return false;
}

__device__ __forceinline__ float token_noise(const SampleParams& P, int b, int pos_flat, int l, int v) {
  if (P.noise_kind == YAPD_NOISE_EXPLICIT) {
    return __ldg(P.gumbel_tok + (int64_t)b * P.gt_stride_req + (int64_t)l * P.gt_stride_pos + v);
  }
  return philox_token_gumbel(P.seed, P.offset, (uint32_t)pos_flat, (uint32_t)v);
}

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
struct Smem {
  uint64_t full[C::NSTAGE];
  float redf[2 * 4 * C::NW];
  double redd[2 * 2 * C::NW];
  int redi[2 * 4 * C::NW];
  int misc[8];
  float miscf[8];
  unsigned long long cand[C::CAP];
  double scan[C::NW + 1];
  alignas(128) unsigned char stage[C::NSTAGE][C::STAGE_BYTES];
};

// Per-thread register tile of one row: NVT vectors of W elements, kept as
// raw 16-byte words (bf16 pairs or fp32).
template <class C>
struct Tile {
  uint4 v[C::NVT];
  __device__ __forceinline__ float get(int k, int i) const {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&v[k]);
    if constexpr (C::BF16) {
      return (i & 1) ? bf16hi(w[i >> 1]) : bf16lo(w[i >> 1]);
    } else {
      return __uint_as_float(w[i]);
    }
  }
  __device__ __forceinline__ void set_neg_inf(int k, int i) {
    uint32_t* w = reinterpret_cast<uint32_t*>(&v[k]);
    if constexpr (C::BF16) {
      if (i & 1) w[i >> 1] = (w[i >> 1] & 0x0000ffffu) | 0xff800000u;
      else w[i >> 1] = (w[i >> 1] & 0xffff0000u) | 0x0000ff80u;
    } else {
      w[i] = 0xff800000u;
    }
  }
  __device__ __forceinline__ void set(int k, int i, float f) {
    uint32_t* w = reinterpret_cast<uint32_t*>(&v[k]);
    if constexpr (C::BF16) {
      const uint32_t h = __float_as_uint(f) >> 16;  // exact: f came from bf16
      if (i & 1) w[i >> 1] = (w[i >> 1] & 0x0000ffffu) | (h << 16);
      else w[i >> 1] = (w[i >> 1] & 0xffff0000u) | h;
    } else {
      w[i] = __float_as_uint(f);
    }
  }
};

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
  if constexpr (C::BF16) {
    const unsigned short h = reinterpret_cast<const unsigned short*>(s)[v + g.head];
    return __uint_as_float((uint32_t)h << 16);
  } else {
    return reinterpret_cast<const float*>(s)[v + g.head];
  }
}

// Load this thread's vectors of a row from the staged copy.  Element v of
// vector k is j*W + i - head with j = tid + k*NT; invalid elements read -inf.
// Returns a bitmask of vectors that contain any invalid or out-of-copy element.
template <class C>
__device__ __forceinline__ uint32_t load_tile(Tile<C>& t, const unsigned char* s, const RowGeom& g, int V) {
  uint32_t edge = 0;
  const int tid = threadIdx.x;
#pragma unroll
  for (int k = 0; k < C::NVT; ++k) {
    const int j = tid + k * C::NT;
    const int v0 = j * C::W - g.head;
    if ((uint32_t)(j * 16) < g.bytes) {
      t.v[k] = *reinterpret_cast<const uint4*>(s + j * 16);
    } else {
      t.v[k] = make_uint4(0, 0, 0, 0);
    }
    const bool interior = v0 >= 0 && v0 + C::W <= g.avail;
    if (!interior) {
      edge |= 1u << k;
#pragma unroll
      for (int i = 0; i < C::W; ++i) {
        const int v = v0 + i;
        if (v < 0 || v >= V) t.set_neg_inf(k, i);
        else if (v >= g.avail) t.set(k, i, load_elem_global<C>(g.row, v));
      }
    }
  }
  return edge;
}

// Same element mapping as `ref_geom` for a row staged with a different head.
template <class C>
__device__ __forceinline__ void load_tile_rephase(Tile<C>& t, const unsigned char* s, const RowGeom& g,
                                                  const RowGeom& ref, int V) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int k = 0; k < C::NVT; ++k) {
    const int j = tid + k * C::NT;
    const int v0 = j * C::W - ref.head;
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      const int v = v0 + i;
      if (v < 0 || v >= V) t.set_neg_inf(k, i);
      else t.set(k, i, load_elem_smem<C>(s, g, v));
    }
  }
}

// ------------------------------------------------------------ worklist

__global__ void worklist_kernel(const int64_t* __restrict__ xt, const uint8_t* __restrict__ is_commit,
                                int B, int L, int64_t mask_id, int dense, int32_t* __restrict__ work,
                                int32_t* __restrict__ count) {
  __shared__ int warp_cnt[32];
  __shared__ int base_s;
  const int total = B * L;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nw = blockDim.x >> 5;
  if (threadIdx.x == 0) base_s = 0;
  __syncthreads();
  for (int p0 = 0; p0 < total; p0 += blockDim.x) {
    const int p = p0 + threadIdx.x;
    bool act = false;
    if (p < total) {
      const int b = p / L;
      act = dense ? true : (is_commit[b] == 0 && xt[p] == mask_id);
    }
    const unsigned bal = __ballot_sync(0xffffffffu, act);
    if (lane == 0) warp_cnt[w] = __popc(bal);
    __syncthreads();
    int off = 0, tot = 0;
    for (int q = 0; q < nw; ++q) {
      const int c = warp_cnt[q];
      off += (q < w) ? c : 0;
      tot += c;
    }
    if (act) work[base_s + off + __popc(bal & ((1u << lane) - 1u))] = p;
    __syncthreads();
    if (threadIdx.x == 0) base_s += tot;
    __syncthreads();
  }
  if (threadIdx.x == 0) *count = base_s;
}

// ------------------------------------------------------------ sample kernel

template <class C>
__device__ __forceinline__ void issue_item(const SampleParams& P, Smem<C>& sm, int stage, int pos) {
  const int b = pos / P.L, l = pos - b * P.L;
  const int64_t base = (int64_t)b * P.stride_req + (int64_t)l * P.stride_pos;
  const RowGeom gc = row_geom<C>(P, base);
  uint32_t bytes = gc.bytes;
  RowGeom gu;
  if (P.nb == 2) {
    gu = row_geom<C>(P, base + P.stride_branch);
    bytes += gu.bytes;
  }
  mbar_arrive_expect_tx(&sm.full[stage], bytes);
  if (gc.bytes) bulk_g2s(sm.stage[stage], gc.src, gc.bytes, &sm.full[stage]);
  if (P.nb == 2 && gu.bytes) bulk_g2s(sm.stage[stage] + C::ROW_SLOT, gu.src, gu.bytes, &sm.full[stage]);
}

template <class C>
__device__ __forceinline__ int item_pos(const SampleParams& P, int idx) {
  return P.n_identity > 0 ? idx : P.work[idx];
}

// Argmax record: (score, tie-break key, vocabulary id) packed so that the
// largest u64 wins.  `tb` is the order key used for exact score ties: for the
// vocabulary-order rule (server/engine.py:548) only the id matters; for the
// sorted-candidate rule (server/engine_ar.py:242) larger vals come first.
struct ArgBest {
  float score;
  float tb;
  int v;
};
__device__ __forceinline__ bool better(float s, float tb, int v, const ArgBest& b, bool use_tb) {
  if (s > b.score) return true;
  if (s < b.score) return false;
  if (s != s) return false;
  if (use_tb && tb != b.tb) return tb > b.tb;
  return v < b.v;
}

// Count and e-mass (double) of the register-resident elements with
// ord_key(key) >= x, restricted to `lo_key` (elements with ord_key < lo_key are
// ignored when lo_key > 0).
template <class C>
__device__ __forceinline__ void count_mass_ge(const float (&key)[C::NS], const float (&e)[C::NS],
                                              int vbase, int V, uint32_t x, int& cnt, double& mass) {
  int c = 0;
  float m = 0.f;
#pragma unroll
  for (int s = 0; s < C::NS; ++s) {
    const int v = vbase + (s / C::W) * C::NT * C::W + (s % C::W);
    const bool in = v >= 0 && v < V && ord_key(key[s]) >= x && key[s] == key[s];
    c += in ? 1 : 0;
    m += in ? e[s] : 0.f;
  }
  cnt = c;
  mass = (double)m;
}

// Sampling with top-k / top-p / min-p / penalty (server/engine_ar.py:230-243
// and the min-p extension).  Returns the chosen vocabulary id.
template <class C>
__device__ __forceinline__ int filtered_select(const SampleParams& P, Smem<C>& sm, BlockRed<C::NW>& red,
                                            const float (&key)[C::NS], int vbase, int b, int pos,
                                            int l, int topk_raw, float top_p, float min_p, float rep,
                                            bool topk_on, bool topp_on, bool minp_on, bool pen_on,
                                            bool noisy) {
  const int tid = threadIdx.x;
  const int V = P.V;
  const int k_eff = topk_on ? topk_raw : V;
  const float rrep = pen_on ? __fdiv_rn(1.0f, rep) : 1.0f;

  // ---- softmax over the candidates: vmax, e = exp(vals - vmax), S ----
  float vm_l = kNegInf;
#pragma unroll
  for (int s = 0; s < C::NS; ++s) vm_l = fmaxf(vm_l, key[s]);
  const float vmax = red.max2(vm_l, 0.f).x;
  float e[C::NS];
  float s_l = 0.f;
#pragma unroll
  for (int s = 0; s < C::NS; ++s) {
    e[s] = ex2_approx(__fmul_rn(__fsub_rn(key[s], vmax), kLog2e));
    if (!(e[s] == e[s])) e[s] = 0.f;
    s_l += e[s];
  }
  const float S = red.sum2(s_l, 0.f).x;

  // ---- candidate threshold: kept (and the top-k set when needed) lie at or above it ----
  float thr = kNegInf;
  int n_c = 0;
  int pick_out = 6;
  {
    // ladder on d = vmax - vals; slot 6 is "everything"
    constexpr int NL = 7;
    const float D[NL] = {1.f, 2.f, 4.f, 8.f, 16.f, 32.f, 3.0e38f};
    float t_m = kNegInf;
    if (minp_on) t_m = fminf(__fsub_rn(__fadd_rn(vmax, logf(min_p)), kMinPMargin), vmax);
    int cnt[NL];
    float mass[NL];
#pragma unroll
    for (int j = 0; j < NL; ++j) {
      cnt[j] = 0;
      mass[j] = 0.f;
    }
    int cnt_m = 0;
#pragma unroll
    for (int s = 0; s < C::NS; ++s) {
      const float d = __fsub_rn(vmax, key[s]);
#pragma unroll
      for (int j = 0; j < NL; ++j) {
        const bool in = d <= D[j];
        cnt[j] += in ? 1 : 0;
        mass[j] += in ? e[s] : 0.f;
      }
      cnt_m += (key[s] >= t_m && minp_on) ? 1 : 0;
    }
    // block totals (counts exact, masses in float)
    int4 c0 = red.sum4i(make_int4(cnt[0], cnt[1], cnt[2], cnt[3]));
    int4 c1 = red.sum4i(make_int4(cnt[4], cnt[5], cnt[6], cnt_m));
    float2 m01 = red.sum2(mass[0], mass[1]);
    float2 m23 = red.sum2(mass[2], mass[3]);
    float2 m45 = red.sum2(mass[4], mass[5]);
    const int ct[NL] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z};
    const float mt[NL] = {m01.x, m01.y, m23.x, m23.y, m45.x, m45.y, S};
    const float need_mass = __fmul_rn(__fmul_rn(top_p, S), 1.0001f);
    int pick = NL - 1;
    if (!topk_on && minp_on) {
      thr = t_m;
      n_c = c1.w;
      pick = -1;
    } else {
#pragma unroll
      for (int j = NL - 1; j >= 0; --j) {
        const bool ok = topk_on ? (ct[j] >= k_eff)
                                : ((topp_on && mt[j] >= need_mass) || (minp_on && vmax - D[j] <= t_m));
        if (ok) pick = j;
      }
      thr = (pick == NL - 1) ? kNegInf : __fsub_rn(vmax, D[pick]);
      n_c = ct[pick];
      // the ladder compares d = vmax - key <= D; keep the same predicate below
    }
    pick_out = pick;
  }
  const int pick = pick_out;
  const float Dpick[7] = {1.f, 2.f, 4.f, 8.f, 16.f, 32.f, 3.0e38f};
  auto in_c = [&](float kv) -> bool {
    if (pick < 0) return kv >= thr;
    return __fsub_rn(vmax, kv) <= Dpick[pick];
  };

  if (n_c <= C::CAP) {
    // ================= small path: compact, sort, resolve exactly =================
    __syncthreads();
    if (tid == 0) sm.misc[0] = 0;
    __syncthreads();
#pragma unroll
    for (int s = 0; s < C::NS; ++s) {
      const int v = vbase + (s / C::W) * C::NT * C::W + (s % C::W);
      const bool in = (v >= 0 && v < V) && in_c(key[s]);
      const unsigned bal = __ballot_sync(0xffffffffu, in);
      if (bal) {
        int basew = 0;
        const int lane = tid & 31;
        if (lane == 0) basew = atomicAdd(&sm.misc[0], __popc(bal));
        basew = __shfl_sync(0xffffffffu, basew, 0);
        if (in) {
          const int at = basew + __popc(bal & ((1u << lane) - 1u));
          if (at < C::CAP) sm.cand[at] = cand_key(key[s], v);
        }
      }
    }
    __syncthreads();
    int nc = sm.misc[0];
    if (nc > C::CAP) nc = C::CAP;
    int npad = 1;
    while (npad < nc) npad <<= 1;
    for (int q = nc + tid; q < npad; q += C::NT) sm.cand[q] = 0ull;
    __syncthreads();
    if (npad <= 32) {
      if (tid < 32) {
        unsigned long long x = tid < npad ? sm.cand[tid] : 0ull;
        x = warp_bitonic_desc(x);
        if (tid < npad) sm.cand[tid] = x;
      }
      __syncthreads();
    } else {
      block_bitonic_desc(sm.cand, npad, C::NT);
    }
    // ---- normaliser: S over all tokens, or over the top-k list ----
    float Sn = S;
    if (topk_on) {
      float part = 0.f;
      for (int q = tid; q < nc && q < k_eff; q += C::NT)
        part += ex2_approx(__fmul_rn(__fsub_rn(cand_val(sm.cand[q]), vmax), kLog2e));
      Sn = red.sum2(part, 0.f).x;
    }
    const float r = __fdiv_rn(1.0f, Sn);
    const float p0 = __fmul_rn(ex2_approx(__fmul_rn(__fsub_rn(cand_val(sm.cand[0]), vmax), kLog2e)), r);
    const float minp_thr = __fmul_rn(min_p, p0);
    // ---- inclusive prefix sums of p in sorted order (double), block scan ----
    constexpr int PER = C::CAP / C::NT;  // candidates per thread
    double pre[PER];
    float pv[PER];
    double run = 0.0;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int q = tid * PER + u;
      float p = 0.f;
      if (q < nc) p = __fmul_rn(ex2_approx(__fmul_rn(__fsub_rn(cand_val(sm.cand[q]), vmax), kLog2e)), r);
      pv[u] = p;
      run += (double)p;
      pre[u] = run;
    }
    // exclusive scan of per-thread totals
    double tot = run;
    const int lane = tid & 31, wid = tid >> 5;
    double incl = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) sm.scan[wid] = incl;
    __syncthreads();
    double woff = 0.0;
    for (int q = 0; q < wid; ++q) woff += sm.scan[q];
    const double toff = woff + incl - tot;
    // ---- keep masks and the penalised, noised score of kept candidates ----
    unsigned long long best = 0ull;  // (score key, -q) max
    bool any_kept = false;
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int q = tid * PER + u;
      if (q >= nc) continue;
      const unsigned long long c = sm.cand[q];
      const float vals = cand_val(c);
      const int v = cand_id(c);
      bool keep = true;
      if (topk_on) keep = keep && (q < k_eff);
      if (topp_on) {
        const float cum = __fsub_rn((float)(toff + pre[u]), pv[u]);
        keep = keep && (cum < top_p);
      }
      if (minp_on) keep = keep && (pv[u] >= minp_thr);
      if (!keep) continue;
      float sc = vals;
      if (pen_on && history_has(P, b, v)) sc = penalize(vals, rep, rrep);
      if (noisy) sc = __fadd_rn(sc, token_noise(P, b, pos, l, v));
      if (!(sc == sc) || sc == kNegInf) continue;
      any_kept = true;
      const unsigned long long rec = ((unsigned long long)ord_key(sc) << 32) | (uint32_t)(0x7fffffff - q);
      best = rec > best ? rec : best;
    }
    (void)any_kept;
    const unsigned long long win = red.max_u64(best);
    const int qwin = (win == 0ull) ? 0 : (0x7fffffff - (int)(uint32_t)win);
    return cand_id(sm.cand[qwin < nc ? qwin : 0]);
  }

  // ================= large path: exact boundaries by bisection over registers =================
  // top-1 (lowest id at vmax) for the "nothing kept" case
  const uint32_t kmax = ord_key(vmax);
  // (i) top-k boundary x_k: largest x with count(ord >= x) >= k
  uint32_t xk = 0u;
  int Jk = 0, tk = 0;
  double Sk = (double)S;
  float rr = __fdiv_rn(1.0f, S);
  if (topk_on) {
    uint32_t lo = 0u, hi = kmax;
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo + 1u) / 2u;
      int c;
      double m;
      count_mass_ge<C>(key, e, vbase, V, mid, c, m);
      int dummy = 0;
      double dm = 0.0;
      red.sum_mixed(m, dm, c, dummy);
      if (c >= k_eff) lo = mid;
      else hi = mid - 1u;
    }
    xk = lo;
    int cg, ce;
    double mg, me;
    count_mass_ge<C>(key, e, vbase, V, xk + 1u, cg, mg);
    count_mass_ge<C>(key, e, vbase, V, xk, ce, me);
    red.sum_mixed(mg, me, cg, ce);
    Jk = k_eff - cg;
    tk = ce - cg;
    const double etie = (double)ex2_approx(__fmul_rn(__fsub_rn(ord_key_inv(xk), vmax), kLog2e));
    Sk = mg + (double)Jk * etie;
    rr = __fdiv_rn(1.0f, (float)Sk);
  }
  // (ii) top-p boundary x_p: smallest x >= xk with G(x) = sum_{ord > x} p < top_p
  uint32_t xp = 0u;
  int Jp = 0x7fffffff;
  bool none_kept = false;
  if (topp_on) {
    if (!(top_p > 0.0f)) {
      none_kept = true;
    } else {
      auto Gp = [&](uint32_t x) -> double {
        int c = 0;
        float m = 0.f;
#pragma unroll
        for (int s = 0; s < C::NS; ++s) {
          const uint32_t o = ord_key(key[s]);
          const bool in = o > x && key[s] == key[s] && (!topk_on || o > xk);
          m += in ? __fmul_rn(e[s], rr) : 0.f;
        }
        double md = (double)m, d2 = 0.0;
        int i2 = 0;
        red.sum_mixed(md, d2, c, i2);
        if (topk_on && x < xk) {
          // ties at xk inside the top-k list also count when x < xk
          int cg, ce;
          double mg, me;
          count_mass_ge<C>(key, e, vbase, V, xk + 1u, cg, mg);
          count_mass_ge<C>(key, e, vbase, V, xk, ce, me);
          red.sum_mixed(mg, me, cg, ce);
          const float etie = ex2_approx(__fmul_rn(__fsub_rn(ord_key_inv(xk), vmax), kLog2e));
          md += (double)Jk * (double)__fmul_rn(etie, rr);
        }
        return md;
      };
      uint32_t lo = topk_on ? xk : 0u, hi = kmax;
      if (Gp(lo) < (double)top_p) {
        xp = lo;
      } else {
        while (hi - lo > 1u) {
          const uint32_t mid = lo + (hi - lo) / 2u;
          if (Gp(mid) < (double)top_p) hi = mid;
          else lo = mid;
        }
        xp = hi;
      }
      // ties at xp: j-th tie (by id) kept iff fl(fl(G + (j+1)p) - p) < top_p
      int cg, ce;
      double mg, me;
      count_mass_ge<C>(key, e, vbase, V, xp + 1u, cg, mg);
      count_mass_ge<C>(key, e, vbase, V, xp, ce, me);
      red.sum_mixed(mg, me, cg, ce);
      const int tp = ce - cg;
      const double G = Gp(xp);
      const float pt = __fmul_rn(ex2_approx(__fmul_rn(__fsub_rn(ord_key_inv(xp), vmax), kLog2e)), rr);
      int lo_j = 0, hi_j = tp;  // first failing j in [0, tp]
      while (lo_j < hi_j) {
        const int mid = (lo_j + hi_j) / 2;
        const float cum = __fsub_rn((float)(G + (double)(mid + 1) * (double)pt), pt);
        if (cum < top_p) lo_j = mid + 1;
        else hi_j = mid;
      }
      Jp = lo_j;
      if (topk_on && xp == xk && Jp > Jk) Jp = Jk;
    }
  }
  // (iii) min-p threshold on p
  const float p0 = __fmul_rn(ex2_approx(__fmul_rn(__fsub_rn(vmax, vmax), kLog2e)), rr);
  const float minp_thr = __fmul_rn(min_p, p0);
  // tie-id limits for partially kept tie groups: keep the J smallest ids
  auto id_limit = [&](uint32_t x, int J) -> int {
    // largest id bound such that count(ord == x && id <= bound) <= J, via bisection
    int lo = -1, hi = V - 1;
    while (lo < hi) {
      const int mid = lo + (hi - lo + 1) / 2;
      int c = 0;
#pragma unroll
      for (int s = 0; s < C::NS; ++s) {
        const int v = vbase + (s / C::W) * C::NT * C::W + (s % C::W);
        c += (v >= 0 && v < V && ord_key(key[s]) == x && v <= mid) ? 1 : 0;
      }
      double a = 0.0, bb = 0.0;
      int z = 0;
      red.sum_mixed(a, bb, c, z);
      if (c <= J) lo = mid;
      else hi = mid - 1;
    }
    return lo;
  };
  int idk = V, idp = V;
  if (topk_on && Jk < tk) idk = id_limit(xk, Jk);
  if (topp_on && !none_kept) {
    int cg, ce;
    double mg, me;
    count_mass_ge<C>(key, e, vbase, V, xp + 1u, cg, mg);
    count_mass_ge<C>(key, e, vbase, V, xp, ce, me);
    red.sum_mixed(mg, me, cg, ce);
    if (Jp < ce - cg) idp = id_limit(xp, Jp);
  }
  // (iv) final argmax over kept: (score desc, vals desc, id asc)
  ArgBest best{kNegInf, kNegInf, 0x7fffffff};
  bool anyk = false;
  if (!none_kept) {
#pragma unroll
    for (int s = 0; s < C::NS; ++s) {
      const int v = vbase + (s / C::W) * C::NT * C::W + (s % C::W);
      if (v < 0 || v >= V) continue;
      const float kv = key[s];
      const uint32_t o = ord_key(kv);
      bool keep = true;
      if (topk_on) keep = keep && (o > xk || (o == xk && v <= idk));
      if (topp_on) keep = keep && (o > xp || (o == xp && v <= idp));
      if (minp_on) keep = keep && (__fmul_rn(e[s], rr) >= minp_thr);
      if (!keep) continue;
      float sc = kv;
      if (pen_on && history_has(P, b, v)) sc = penalize(kv, rep, rrep);
      if (noisy) sc = __fadd_rn(sc, token_noise(P, b, pos, l, v));
      if (!(sc == sc) || sc == kNegInf) continue;
      anyk = true;
      if (better(sc, kv, v, best, true)) best = {sc, kv, v};
    }
  }
  const uint32_t sk = anyk ? ord_key(best.score) : 0u;
  const unsigned long long w1 = red.max_u64(((unsigned long long)sk << 32) | (anyk ? ord_key(best.tb) : 0u));
  if (w1 == 0ull) {
    // nothing kept: the first sorted candidate (largest vals, lowest id)
    int c_id = 0x7fffffff;
#pragma unroll
    for (int s = 0; s < C::NS; ++s) {
      const int v = vbase + (s / C::W) * C::NT * C::W + (s % C::W);
      if (v >= 0 && v < V && ord_key(key[s]) == kmax && v < c_id) c_id = v;
    }
    const unsigned long long w = red.max_u64((unsigned long long)(uint32_t)(0x7fffffff - c_id));
    const int id = 0x7fffffff - (int)(uint32_t)w;
    return (id >= 0 && id < V) ? id : 0;
  }
  const bool tie = anyk && ((((unsigned long long)sk << 32) | ord_key(best.tb)) == w1);
  const unsigned long long w2 = red.max_u64(tie ? (unsigned long long)(uint32_t)(0x7fffffff - best.v) : 0ull);
  const int id = 0x7fffffff - (int)(uint32_t)w2;
  return (id >= 0 && id < V) ? id : 0;
}

template <class C>
__device__ __forceinline__ void process_item(const SampleParams& P, Smem<C>& sm, BlockRed<C::NW>& red,
                                          int stage, int pos) {
  const int tid = threadIdx.x;
  const int V = P.V;
  const int b = pos / P.L, l = pos - b * P.L;
  const int64_t base = (int64_t)b * P.stride_req + (int64_t)l * P.stride_pos;
  const RowGeom gc = row_geom<C>(P, base);
  const unsigned char* sc = sm.stage[stage];
  const unsigned char* su = sm.stage[stage] + C::ROW_SLOT;
  const bool cfg = (P.nb == 2);

  // ---- registers: cond and uncond tiles ----
  Tile<C> tc, tu;
  const uint32_t edge = load_tile<C>(tc, sc, gc, V);
  RowGeom gu;
  if (cfg) {
    gu = row_geom<C>(P, base + P.stride_branch);
    if (gu.head == gc.head) load_tile<C>(tu, su, gu, V);
    else load_tile_rephase<C>(tu, su, gu, gc, V);
  }

  // ---- sampling parameters ----
  const float T = param_f(P.temperature, P.temperature_s, b);
  const int topk_raw = param_i(P.top_k, P.top_k_s, b);
  const float top_p = param_f(P.top_p, P.top_p_s, b);
  const float min_p = param_f(P.min_p, P.min_p_s, b);
  const float rep = param_f(P.rep_penalty, P.rep_penalty_s, b);
  const bool has_hist = P.history_kind != YAPD_HISTORY_NONE && P.history != nullptr;
  const bool topk_on = topk_raw > 0 && topk_raw < V;
  const bool topp_on = top_p < 1.0f;
  const bool minp_on = min_p > 0.0f;
  const bool pen_on = has_hist && rep != 1.0f;
  const bool filtered = topk_on || topp_on || minp_on || pen_on;
  const bool noisy = T > 0.0f || !P.zero_temp_greedy;
  const bool scale = T > 0.0f;
  const float rT = scale ? __fdiv_rn(1.0f, T) : 1.0f;

  // ---- P1: row maxima ----
  float mc_l = kNegInf, mu_l = kNegInf;
#pragma unroll
  for (int k = 0; k < C::NVT; ++k)
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      mc_l = fmaxf(mc_l, tc.get(k, i));
      if (cfg) mu_l = fmaxf(mu_l, tu.get(k, i));
    }
  const float2 mx = red.max2(mc_l, mu_l);
  const float mc = mx.x, mu = mx.y;

  // ---- P2: sums of exp(x - max) ----
  float sc_l = 0.f, su_l = 0.f;
#pragma unroll
  for (int k = 0; k < C::NVT; ++k)
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      sc_l += ex2_approx(__fmul_rn(__fsub_rn(tc.get(k, i), mc), kLog2e));
      if (cfg) su_l += ex2_approx(__fmul_rn(__fsub_rn(tu.get(k, i), mu), kLog2e));
    }
  const float2 sm2 = red.sum2(sc_l, su_l);
  const float Sc = sm2.x, Su = sm2.y;
  const float lc = logf(Sc), lu = logf(Su);

  // ---- P3: guided / T for every element (exact op order of the reference) ----
  float key[C::NS];
#pragma unroll
  for (int k = 0; k < C::NVT; ++k)
#pragma unroll
    for (int i = 0; i < C::W; ++i) {
      float g;
      if (cfg) {
        const float lsc = __fsub_rn(__fsub_rn(tc.get(k, i), mc), lc);
        const float lsu = __fsub_rn(__fsub_rn(tu.get(k, i), mu), lu);
        g = __fadd_rn(lsc, __fmul_rn(P.cfg_w, __fsub_rn(lsc, lsu)));
      } else {
        g = tc.get(k, i);
      }
      key[k * C::W + i] = scale ? div_rn(g, T, rT) : g;
    }
  if (edge) {
#pragma unroll
    for (int k = 0; k < C::NVT; ++k) {
      if (!((edge >> k) & 1u)) continue;
      const int v0 = (tid + k * C::NT) * C::W - gc.head;
#pragma unroll
      for (int i = 0; i < C::W; ++i) {
        const int v = v0 + i;
        if (v < 0 || v >= V) key[k * C::W + i] = kNegInf;
      }
    }
  }
  const int vbase = tid * C::W - gc.head;  // element id of slot (k, i) = vbase + k*NT*W + i

  // torch orders NaN above every number (sort, topk and argmax), so a row with
  // a NaN value samples its lowest-id NaN token whatever the filters are.
  bool nan_l = false;
#pragma unroll
  for (int s = 0; s < C::NS; ++s) nan_l |= !(key[s] == key[s]);
  int chosen = 0;
  if (__syncthreads_or(nan_l)) {
    int first_nan = 0x7fffffff;
#pragma unroll
    for (int s = 0; s < C::NS; ++s) {
      const int v = vbase + (s / C::W) * C::NT * C::W + (s % C::W);
      if (v >= 0 && v < V && !(key[s] == key[s]) && v < first_nan) first_nan = v;
    }
    const unsigned long long w = red.max_u64((unsigned long long)(uint32_t)(0x7fffffff - first_nan));
    chosen = 0x7fffffff - (int)(uint32_t)w;
  } else if (!filtered) {
    // ---- unfiltered: argmax(guided / T + G) in vocabulary order (engine.py:546-550) ----
    ArgBest best{kNegInf, 0.f, 0x7fffffff};
#pragma unroll
    for (int k = 0; k < C::NVT; ++k)
#pragma unroll
      for (int i = 0; i < C::W; ++i) {
        const int v = vbase + k * C::NT * C::W + i;
        if (v < 0 || v >= V) continue;
        float s = key[k * C::W + i];
        if (noisy) s = __fadd_rn(s, token_noise(P, b, pos, l, v));
        if (better(s, 0.f, v, best, false)) best = {s, 0.f, v};
      }
    // block argmax: largest score, then smallest id; NaN scores lose
    const uint32_t sk = (best.score == best.score) ? ord_key(best.score) : 0u;
    const unsigned long long packed =
        ((unsigned long long)sk << 32) | (uint32_t)(0x7fffffff - (best.v > V ? V : best.v));
    const unsigned long long win = red.max_u64(packed);
    chosen = cand_id(win);
    if (chosen >= V || chosen < 0) chosen = 0;
  } else if (!topk_on && !topp_on && !minp_on) {
    // ---- penalty only: every token kept; order ties by (vals desc, id asc) ----
    const float rrep = __fdiv_rn(1.0f, rep);
    ArgBest best{kNegInf, kNegInf, 0x7fffffff};
#pragma unroll
    for (int k = 0; k < C::NVT; ++k)
#pragma unroll
      for (int i = 0; i < C::W; ++i) {
        const int v = vbase + k * C::NT * C::W + i;
        if (v < 0 || v >= V) continue;
        const float kv = key[k * C::W + i];
        float s = history_has(P, b, v) ? penalize(kv, rep, rrep) : kv;
        if (noisy) s = __fadd_rn(s, token_noise(P, b, pos, l, v));
        if (better(s, kv, v, best, true)) best = {s, kv, v};
      }
    // two-stage reduction: first the best score, then the order key among equal scores
    const uint32_t sk = (best.score == best.score) ? ord_key(best.score) : 0u;
    const unsigned long long w1 = red.max_u64(((unsigned long long)sk << 32) | ord_key(best.tb));
    const bool tie = ((unsigned long long)sk << 32 | ord_key(best.tb)) == w1;
    const unsigned long long w2 =
        red.max_u64(tie ? (unsigned long long)(uint32_t)(0x7fffffff - best.v) : 0ull);
    chosen = 0x7fffffff - (int)(uint32_t)w2;
    if (chosen >= V || chosen < 0) chosen = 0;
  } else {
    chosen = filtered_select<C>(P, sm, red, key, vbase, b, pos, l, topk_raw, top_p, min_p, rep,
                                topk_on, topp_on, minp_on, pen_on, noisy);
  }

  if (chosen < 0 || chosen >= V) {
    if (tid == 0) atomicOr(P.status, (unsigned)YAPD_STATUS_INTERNAL);
    chosen = 0;
  }
  // ---- PMI of the chosen token (engine.py:553-558) ----
  if (tid == 0) {
    P.sampled[pos] = chosen;
    if (P.want_pmi) {
      const float cv = load_elem_smem<C>(sc, gc, chosen);
      const float rc = __fdiv_rn(1.0f, Sc);
      const float pc = __fmul_rn(expf(__fsub_rn(cv, mc)), rc);
      const float lp = __ldg(P.log_prior + chosen);
      const float lpl = __fmul_rn(P.pmi_lambda, lp);
      float pmi = __fsub_rn(logf(fmaxf(pc, 1e-8f)), lpl);
      if (cfg) {
        const float uv = load_elem_smem<C>(su, gu, chosen);
        const float ru = __fdiv_rn(1.0f, Su);
        const float pu = __fmul_rn(expf(__fsub_rn(uv, mu)), ru);
        const float pmi_u = __fsub_rn(logf(fmaxf(pu, 1e-8f)), lpl);
        pmi = __fsub_rn(__fmul_rn(P.cfg_1pw, pmi), __fmul_rn(P.cfg_w, pmi_u));
      }
      P.pmi[pos] = pmi;
    }
  }
}

}  // namespace yapd

namespace yapd {

template <class C>
__global__ void __launch_bounds__(C::NT, C::MINB) sample_kernel(const SampleParams P) {
  extern __shared__ unsigned char smem_raw[];
  Smem<C>& sm = *reinterpret_cast<Smem<C>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  const int n_items = P.n_identity > 0 ? P.n_identity : *P.work_count;
  const int first = blockIdx.x, stride = gridDim.x;
  if (first >= n_items) return;
  const int n_my = (n_items - first + stride - 1) / stride;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE; ++s) mbar_init(&sm.full[s], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NSTAGE && s < n_my; ++s)
      issue_item<C>(P, sm, s, item_pos<C>(P, first + s * stride));
  }
  BlockRed<C::NW> red{sm.redf, sm.redd, sm.redi, 0};
  for (int it = 0; it < n_my; ++it) {
    const int stage = it % C::NSTAGE;
    const uint32_t parity = (uint32_t)(it / C::NSTAGE) & 1u;
    const bool ok = mbar_wait_bounded(&sm.full[stage], parity, kWaitLimitNs);
    if (__syncthreads_or(!ok)) {
      // A copy did not land in time: record it, give the copies still in
      // flight a bounded chance to finish, and leave without touching them.
      if (threadIdx.x == 0) {
        atomicOr(P.status, (unsigned)YAPD_STATUS_WAIT_TIMEOUT);
        for (int q = it; q < n_my && q < it + C::NSTAGE; ++q)
          (void)mbar_wait_bounded(&sm.full[q % C::NSTAGE], (uint32_t)(q / C::NSTAGE) & 1u, kWaitLimitNs);
      }
      __syncthreads();
      return;
    }
    process_item<C>(P, sm, red, stage, item_pos<C>(P, first + it * stride));
    __syncthreads();
    if (threadIdx.x == 0 && it + C::NSTAGE < n_my) {
      fence_proxy_async_smem();
      issue_item<C>(P, sm, stage, item_pos<C>(P, first + (it + C::NSTAGE) * stride));
    }
  }
}

// Positions that are not sampled (sparse mode) report sampled = -1, pmi = NaN.
__global__ void init_outputs_kernel(const int64_t* __restrict__ xt, const uint8_t* __restrict__ is_commit,
                                    int B, int L, int64_t mask_id, int dense, int32_t* __restrict__ sampled,
                                    float* __restrict__ pmi) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p >= B * L || dense) return;
  const int b = p / L;
  if (!(is_commit[b] == 0 && xt[p] == mask_id)) {
    sampled[p] = -1;
    pmi[p] = __int_as_float(0x7fc00000);
  }
}

struct UnmaskParams {
  const int64_t* xt;
  const int64_t* k_step;
  const uint8_t* is_commit;
  const int64_t* sched_t;
  const float* q_t;
  const int32_t* sampled;
  float* pmi;
  const float* gumbel_pos;
  int noise_kind;
  uint64_t seed, offset;
  int B, L, K;
  int64_t mask_id, stop_id;
  int pos_noise, use_quantile;
  int64_t* xt_out;
  int32_t* n_unmask;
  int32_t* n_mask_after;
  uint8_t* hit_eos;
  int64_t* k_step_out;
  uint8_t* is_commit_out;
};

// Total order used to rank PMI: NaN above +inf (torch's sort order).
__device__ __forceinline__ uint32_t rank_key(float f) {
  return (f != f) ? 0xffffffffu : ord_key(f);
}

// One warp per request: server/engine.py:559-612.
__global__ void unmask_kernel(const UnmaskParams U) {
  const int lane = threadIdx.x & 31;
  const int b = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (b >= U.B) return;
  const int L = U.L, K = U.K;
  const bool in = lane < L;
  const int p = b * L + lane;
  const int64_t x = in ? U.xt[p] : 0;
  const bool is_mask = in && x == U.mask_id;
  const bool commit = U.is_commit[b] != 0;
  const bool denoise = !commit;
  const int64_t ks = U.k_step[b];
  int kc = (int)(ks < (int64_t)(K - 1) ? ks : (int64_t)(K - 1));
  if (kc < 0) kc = 0;
  // ranked PMI: position noise on masked positions (engine.py:559-561)
  float pm = 0.f;
  if (is_mask) {
    pm = U.pmi[p];
    if (U.pos_noise) {
      const float gn = (U.noise_kind == YAPD_NOISE_EXPLICIT)
                           ? U.gumbel_pos[p]
                           : philox_position_gumbel(U.seed, U.offset, (uint32_t)p);
      pm = __fadd_rn(pm, gn);
    }
  }
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
  const float tau = __fadd_rn(v_lo, __fmul_rn(__fsub_rn(pq, (float)lo), __fsub_rn(v_hi, v_lo)));
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
  if (denoise && do_un) xf = (int64_t)U.sampled[p];
  if (in) {
    U.xt_out[p] = xf;
    if (is_mask) U.pmi[p] = pm;
  }
  const int n_after = __popc(__ballot_sync(0xffffffffu, in && xf == U.mask_id));
  const bool eos = __any_sync(0xffffffffu, in && xf == U.stop_id);
  if (lane == 0) {
    const int64_t k_new = denoise ? ks + 1 : ks;
    const int64_t k_fin = commit ? 0 : k_new;
    const bool to_commit = denoise && !eos && (n_after == 0 || k_fin >= (int64_t)K);
    U.n_unmask[b] = denoise ? n_un : 0;
    U.n_mask_after[b] = n_after;
    U.hit_eos[b] = eos ? 1 : 0;
    U.k_step_out[b] = k_fin;
    U.is_commit_out[b] = to_commit ? 1 : 0;
  }
}

// ---------------------------------------------------------------- host side

template <class C>
constexpr size_t smem_bytes() {
  return sizeof(Smem<C>) + 128;
}

struct DevInfo {
  int sms = 0;
  int occ_bf16 = 0;
  int occ_f32 = 0;
  bool init = false;
};

static DevInfo g_dev[64];

static int device_info(DevInfo** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return YAPD_ERR_NO_DEVICE;
  DevInfo& d = g_dev[dev];
  if (!d.init) {
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      return YAPD_ERR_NO_DEVICE;
    if (cudaFuncSetAttribute(sample_kernel<CfgBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes<CfgBF16>()) != cudaSuccess)
      return YAPD_ERR_LAUNCH;
    if (cudaFuncSetAttribute(sample_kernel<CfgF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_bytes<CfgF32>()) != cudaSuccess)
      return YAPD_ERR_LAUNCH;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_bf16, sample_kernel<CfgBF16>, CfgBF16::NT,
                                                      smem_bytes<CfgBF16>()) != cudaSuccess)
      return YAPD_ERR_LAUNCH;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&d.occ_f32, sample_kernel<CfgF32>, CfgF32::NT,
                                                      smem_bytes<CfgF32>()) != cudaSuccess)
      return YAPD_ERR_LAUNCH;
    if (d.occ_bf16 < 1 || d.occ_f32 < 1) return YAPD_ERR_LAUNCH;
    d.init = true;
  }
  *out = &d;
  return YAPD_OK;
}

static int fill_sampling(SampleParams& P, const yapd_sampling& s, const yapd_noise& n) {
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
  if (s.history_kind != YAPD_HISTORY_NONE && (!s.history || s.history_stride <= 0))
    return YAPD_ERR_NULL_POINTER;
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

static int launch_sample(const SampleParams& P, int dtype, int max_items, cudaStream_t st) {
  DevInfo* d = nullptr;
  int rc = device_info(&d);
  if (rc != YAPD_OK) return rc;
  if (dtype == YAPD_DTYPE_BF16) {
    int grid = d->sms * d->occ_bf16;
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    sample_kernel<CfgBF16><<<grid, CfgBF16::NT, smem_bytes<CfgBF16>(), st>>>(P);
  } else {
    int grid = d->sms * d->occ_f32;
    if (grid > max_items) grid = max_items;
    if (grid < 1) grid = 1;
    sample_kernel<CfgF32><<<grid, CfgF32::NT, smem_bytes<CfgF32>(), st>>>(P);
  }
  return cudaGetLastError() == cudaSuccess ? YAPD_OK : YAPD_ERR_LAUNCH;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

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

size_t yapd_select_workspace_size(int32_t B, int32_t L) {
  if (B <= 0 || L <= 0) return 256;
  return 256 + align256((size_t)B * (size_t)L * sizeof(int32_t));
}

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
  if (!a) return YAPD_ERR_NULL_POINTER;
  if (a->B <= 0 || a->L <= 0 || a->L > YAPD_MAX_L || a->V <= 0 || a->K <= 0 ||
      (a->nb != 1 && a->nb != 2))
    return YAPD_ERR_BAD_SHAPE;
  if (a->V > YAPD_MAX_V) return YAPD_ERR_V_TOO_LARGE;
  if ((int64_t)a->B * a->L > (1 << 30)) return YAPD_ERR_BAD_SHAPE;
  if (a->logits_dtype != YAPD_DTYPE_F32 && a->logits_dtype != YAPD_DTYPE_BF16) return YAPD_ERR_BAD_DTYPE;
  if (!a->logits || !a->xt || !a->k_step || !a->is_commit || !a->log_prior || !a->sched_t || !a->q_t ||
      !a->xt_out || !a->sampled || !a->pmi || !a->n_unmask || !a->n_mask_after || !a->hit_eos ||
      !a->k_step_out || !a->is_commit_out)
    return YAPD_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(a->logits) & 15u) != 0) return YAPD_ERR_MISALIGNED;
  if (a->stride_req < 0 || a->stride_branch < 0 || a->stride_pos < 0) return YAPD_ERR_BAD_SHAPE;
  const int64_t last = (int64_t)(a->B - 1) * a->stride_req + (int64_t)(a->nb - 1) * a->stride_branch +
                       (int64_t)(a->L - 1) * a->stride_pos + a->V;
  if (a->logits_numel < last) return YAPD_ERR_BAD_SHAPE;
  if (!a->workspace || a->workspace_bytes < yapd_select_workspace_size(a->B, a->L)) return YAPD_ERR_WORKSPACE;
  if (a->noise.kind == YAPD_NOISE_EXPLICIT && a->pos_noise && !a->noise.gumbel_pos)
    return YAPD_ERR_NULL_POINTER;

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
  P.V = a->V;
  int rc = fill_sampling(P, a->sampling, a->noise);
  if (rc != YAPD_OK) return rc;
  char* ws = static_cast<char*>(a->workspace);
  P.status = reinterpret_cast<uint32_t*>(ws);
  P.work_count = reinterpret_cast<int32_t*>(ws + 4);
  P.work = reinterpret_cast<int32_t*>(ws + 256);
  P.n_identity = 0;
  P.log_prior = a->log_prior;
  P.cfg_w = a->cfg_scale;
  P.cfg_1pw = a->cfg_one_plus;
  P.pmi_lambda = a->pmi_lambda;
  P.want_pmi = 1;
  P.sampled = a->sampled;
  P.pmi = a->pmi;

  cudaStream_t st = (cudaStream_t)stream;
  const int total = a->B * a->L;
  worklist_kernel<<<1, 1024, 0, st>>>(a->xt, a->is_commit, a->B, a->L, a->mask_id, a->dense,
                                      reinterpret_cast<int32_t*>(ws + 256),
                                      reinterpret_cast<int32_t*>(ws + 4));
  init_outputs_kernel<<<(total + 255) / 256, 256, 0, st>>>(a->xt, a->is_commit, a->B, a->L, a->mask_id,
                                                           a->dense, a->sampled, a->pmi);
  if (cudaGetLastError() != cudaSuccess) return YAPD_ERR_LAUNCH;
  rc = launch_sample(P, a->logits_dtype, total, st);
  if (rc != YAPD_OK) return rc;

  UnmaskParams U{};
  U.xt = a->xt;
  U.k_step = a->k_step;
  U.is_commit = a->is_commit;
  U.sched_t = a->sched_t;
  U.q_t = a->q_t;
  U.sampled = a->sampled;
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
  U.xt_out = a->xt_out;
  U.n_unmask = a->n_unmask;
  U.n_mask_after = a->n_mask_after;
  U.hit_eos = a->hit_eos;
  U.k_step_out = a->k_step_out;
  U.is_commit_out = a->is_commit_out;
  unmask_kernel<<<(a->B + 3) / 4, 128, 0, st>>>(U);
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
  P.V = a->V;
  int rc = fill_sampling(P, a->sampling, a->noise);
  if (rc != YAPD_OK) return rc;
  P.status = static_cast<uint32_t*>(a->workspace);
  P.work = nullptr;
  P.work_count = nullptr;
  P.n_identity = a->R;
  P.log_prior = nullptr;
  P.want_pmi = 0;
  P.sampled = a->sampled;
  P.pmi = nullptr;
  return launch_sample(P, a->logits_dtype, a->R, (cudaStream_t)stream);
}

}  // extern "C"
