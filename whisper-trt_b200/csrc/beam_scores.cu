// The scoring half of a beam-search step: each row's masked log-softmax plus its cumulative log-probability (the
// K x V candidate scores of its window), each window's no-speech probability, and each window's best 2K
// candidates -- the parents and tokens wt_beam_update consumes.
//
// Semantics: the reference's search.py:283-289 (_choose: suppressed tokens, begin-suppressed ones at a window's
// first step), :313-338 (_timestamp_rules, CTranslate2's ApplyTimestampRules), :369-371 (scores + topk(2K)) and
// :259-260 (no-speech probability); fused there as beam_kernels.py:36-135 (_scores_kernel) + torch.topk.
//
// B200 design: a thread-block cluster of 4 CTAs per row, each CTA a quarter of the vocabulary, exchanging its
// partial maxima, sums and best candidates through distributed shared memory (no global round trips). Coalesced
// sweeps over the slice, 8 independent loads in flight per thread: from HBM the maxima (raw, masked, masked
// timestamps, masked text); then from L2 the sums of exponentials, the scores (written out if asked for) with each
// thread's best one, and -- against a threshold that keeps every one of the row's best 2K -- the few candidates,
// from which one warp picks the CTA's best 2K and rank 0 the row's, written to the workspace;
// the row CTA of a window that arrives last (an atomic count, no waiting) merges the window's K lists into its
// best 2K. Ordering is (score descending, candidate index ascending) everywhere, so equal scores come out in
// index order.
#include <cooperative_groups.h>

#include "common.cuh"

namespace wt {
namespace {

constexpr int kScoreThreads = 256;
constexpr int kScoreCluster = 4;  // CTAs per row (a thread-block cluster exchanging through shared memory)
constexpr int kScoreWarps = kScoreThreads / 32;
constexpr float kLowest = -3.40282346638528859812e+38f;  // the lowest finite float (the reference's LOWEST)

constexpr int kNoCand = 0x7fffffff;  // the index of an empty list entry (after every candidate)

// candidate indices (beam * V + token) fit in 32 bits: beams * vocab < 2^31 is checked at the entry point
__device__ __forceinline__ bool better(float s, int i, float s2, int i2) {
  return s > s2 || (s == s2 && i < i2);
}

// Insert (s, i) into a register list sorted best first (KK entries).
template <int KK>
__device__ __forceinline__ void insert(float (&ls)[KK], int (&li)[KK], float s, int i) {
  if (!better(s, i, ls[KK - 1], li[KK - 1])) return;
  ls[KK - 1] = s;
  li[KK - 1] = i;
#pragma unroll
  for (int j = KK - 1; j > 0; --j) {
    if (better(ls[j], li[j], ls[j - 1], li[j - 1])) {
      const float ts = ls[j];
      ls[j] = ls[j - 1];
      ls[j - 1] = ts;
      const int ti = li[j];
      li[j] = li[j - 1];
      li[j - 1] = ti;
    }
  }
}

// kk rounds of a warp-wide selection over the lanes' sorted lists (each lane offers its head): the warp's best kk,
// best first, in every lane's (out_s, out_i)[0 .. kk).
template <int KK>
__device__ __forceinline__ void warp_select(float (&ls)[KK], int (&li)[KK], int kk, float (&out_s)[KK],
                                            int (&out_i)[KK]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < KK; ++k) {
    if (k >= kk) break;
    float s = ls[0];
    int i = li[0];
    int who = lane;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
      const int w2 = __shfl_xor_sync(0xffffffffu, who, o);
      if (better(s2, i2, s, i)) {
        s = s2;
        i = i2;
        who = w2;
      }
    }
    out_s[k] = s;
    out_i[k] = i;
    if (who == lane) {  // pop the head
#pragma unroll
      for (int j = 0; j < KK - 1; ++j) {
        ls[j] = ls[j + 1];
        li[j] = li[j + 1];
      }
      ls[KK - 1] = -__builtin_huge_valf();
      li[KK - 1] = kNoCand;
    }
  }
}

__device__ __forceinline__ float block_reduce(float x, float *red, bool is_max) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float y = __shfl_xor_sync(0xffffffffu, x, o);
    x = is_max ? fmaxf(x, y) : x + y;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = x;
  __syncthreads();
  x = lane < kScoreWarps ? red[lane] : (is_max ? -__builtin_huge_valf() : 0.f);
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float y = __shfl_xor_sync(0xffffffffu, x, o);
    x = is_max ? fmaxf(x, y) : x + y;
  }
  return x;
}

constexpr int kUnroll = 16;  // elements per thread per chunk: their loads are all in flight at once
constexpr int kGather = 128;  // candidates of a row the cluster's rank 0 ranks directly (more: the exact path)

constexpr float kLog2e = 1.4426950408889634f;

// e^x as 2^(x log2 e) on the special-function unit (ex2.approx: ~2^-22 relative; e^-inf = 0)
__device__ __forceinline__ float fexp(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * kLog2e));
  return y;
}

// An online (max, sum of e^(x - max)) state.
struct Lse {
  float m, s;
};
__device__ __forceinline__ Lse lse_merge(Lse a, Lse b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -__builtin_huge_valf()) return a;
  return Lse{m, a.s * fexp(a.m - m) + b.s * fexp(b.m - m)};
}
// fold a chunk of U values (invalid ones -inf) into the state: one rescale per chunk
template <int U>
__device__ __forceinline__ void lse_chunk(Lse &a, const float (&x)[U]) {
  float cm = x[0];
#pragma unroll
  for (int u = 1; u < U; ++u) cm = fmaxf(cm, x[u]);
  const float m = fmaxf(a.m, cm);
  if (m == -__builtin_huge_valf()) return;
  float acc = a.s * fexp(a.m - m);
#pragma unroll
  for (int u = 0; u < U; ++u) acc += fexp(x[u] - m);
  a.m = m;
  a.s = acc;
}
__device__ __forceinline__ Lse block_lse(Lse x, float *red) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1)
    x = lse_merge(x, Lse{__shfl_xor_sync(0xffffffffu, x.m, o), __shfl_xor_sync(0xffffffffu, x.s, o)});
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) {
    red[2 * warp] = x.m;
    red[2 * warp + 1] = x.s;
  }
  __syncthreads();
  x = lane < kScoreWarps ? Lse{red[2 * lane], red[2 * lane + 1]} : Lse{-__builtin_huge_valf(), 0.f};
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1)
    x = lse_merge(x, Lse{__shfl_xor_sync(0xffffffffu, x.m, o), __shfl_xor_sync(0xffffffffu, x.s, o)});
  return x;
}

// The logits and suppress / begin flags of one chunk: element u of the chunk is v = 2 * (p0 + (u / 2) * threads +
// tid) + u % 2 (pairs of consecutive tokens; each thread visits its elements in increasing order). VEC: the row
// and the flags allow 8-byte / 2-byte pair loads. Past `hi`: x = -inf, flags 0. The begin flags are read only at a
// window's first step (`first`), where they apply.
template <bool VEC, bool CHECK = true>
__device__ __forceinline__ void load_chunk(const float *x, const uint8_t *sup, const uint8_t *beg, int p0, int hi,
                                           bool first, float (&xv)[kUnroll], bool (&su)[kUnroll],
                                           bool (&be)[kUnroll]) {
#pragma unroll
  for (int j = 0; j < kUnroll / 2; ++j) {
    const int v = 2 * (p0 + j * kScoreThreads + static_cast<int>(threadIdx.x));
    if (VEC && (!CHECK || v + 1 < hi)) {
      const float2 xx = __ldg(reinterpret_cast<const float2 *>(x + v));
      const unsigned short sp = __ldg(reinterpret_cast<const unsigned short *>(sup + v));
      const unsigned short bp = first ? __ldg(reinterpret_cast<const unsigned short *>(beg + v)) : 0;
      xv[2 * j] = xx.x;
      xv[2 * j + 1] = xx.y;
      su[2 * j] = (sp & 0xff) != 0;
      su[2 * j + 1] = (sp >> 8) != 0;
      be[2 * j] = (bp & 0xff) != 0;
      be[2 * j + 1] = (bp >> 8) != 0;
    } else {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const bool in = v + h < hi;
        xv[2 * j + h] = in ? __ldg(x + v + h) : -__builtin_huge_valf();
        su[2 * j + h] = in && __ldg(sup + v + h) != 0;
        be[2 * j + h] = in && first && __ldg(beg + v + h) != 0;
      }
    }
  }
}
// The logits alone of one chunk (pairs when VEC), -inf past hi.
template <bool VEC>
__device__ __forceinline__ void load_logits(const float *x, int p0, int hi, float (&xv)[kUnroll]) {
#pragma unroll
  for (int j = 0; j < kUnroll / 2; ++j) {
    const int v = 2 * (p0 + j * kScoreThreads + static_cast<int>(threadIdx.x));
    if (VEC && v + 1 < hi) {
      const float2 xx = __ldg(reinterpret_cast<const float2 *>(x + v));
      xv[2 * j] = xx.x;
      xv[2 * j + 1] = xx.y;
    } else {
      xv[2 * j] = v < hi ? __ldg(x + v) : -__builtin_huge_valf();
      xv[2 * j + 1] = v + 1 < hi ? __ldg(x + v + 1) : -__builtin_huge_valf();
    }
  }
}
__device__ __forceinline__ int chunk_v(int p0, int u) {
  return 2 * (p0 + (u / 2) * kScoreThreads + static_cast<int>(threadIdx.x)) + u % 2;
}

struct ScoreArgs {
  const float *logits;
  const uint8_t *suppress, *begin;
  const int64_t *t, *hist, *max_initial;
  const float *cum;
  const uint8_t *sampling;  // [B] or null: a sampled window's rows score without their cumulative log-probability
  float *scores, *ns, *top_s;
  int64_t *top_i;
  float *row_s;  // workspace: [N, kk] row lists
  int *row_i;    // workspace: [N, kk]
  int *counters; // workspace: [B]
  int K, V, T, kk, cap, timestamps, no_speech, nots, tsb, eot;
};

// The cluster's shared exchange area of one CTA (read by the others through distributed shared memory).
template <int KK>
struct Exchange {
  float red[8];               // this CTA's (max, sum) of the raw, masked and masked-timestamp logits, text maximum
  float wm_s[kScoreWarps];    // each warp's best masked logit (its threads' champions' best) and its index
  int wm_i[kScoreWarps];
  int n_cand;                 // candidates in this CTA's buffer (> cap: it overflowed)
  float ls[KK];               // this CTA's best kk (the exact path)
  int li[KK];
};

// One cluster of kScoreCluster CTAs per row, each CTA a contiguous slice of the vocabulary. TS: timestamp rules.
template <int KK, bool TS>
__global__ void __launch_bounds__(kScoreThreads, 4) beam_scores_kernel(const ScoreArgs a) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  __shared__ float red[2 * kScoreWarps];
  __shared__ float wl_s[kScoreWarps][KK];
  __shared__ int wl_i[kScoreWarps][KK];
  __shared__ long long ts_state[4];  // last, latest, flags, max_init
  __shared__ int is_last, n_cand;
  __shared__ Exchange<KK> ex;
  extern __shared__ unsigned char dyn[];
  float *cand_s = reinterpret_cast<float *>(dyn);
  int *cand_i = reinterpret_cast<int *>(dyn + static_cast<size_t>(a.cap) * sizeof(float));
  const int rank = static_cast<int>(cluster.block_rank());
  const int r = blockIdx.x / kScoreCluster, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = a.K, V = a.V, b = r / K;
  const int per = ((V + kScoreCluster - 1) / kScoreCluster + 1) & ~1;  // (even: slices start on a pair)
  const int lo = min(V, rank * per), hi = min(V, lo + per);

  pdl_wait();
  pdl_launch_dependents();

  const long long tw = a.t[b];
  const bool first = tw == 0;
  // the timestamp rules' state of this row (search.py:320-333): its last two tokens and latest timestamp
  bool first_ts = false, both = false, pair = false, fresh = false, check = false;
  long long last = 0, latest = 0, max_init = 0;
  if (tid == 0) n_cand = 0;
  if (TS) {
    if (warp == 0) {
      const long long g = tw > 0 ? tw : 0;
      const int64_t *h = a.hist + static_cast<size_t>(r) * a.T;
      int at = -1;
      for (int j = lane; j < a.T && j < g; j += 32)
        if (h[j] >= a.tsb) at = j;  // (increasing j: the lane's latest)
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) at = max(at, __shfl_xor_sync(0xffffffffu, at, o));
      if (lane == 0) {
        const long long ls = g >= 1 ? h[min(g - 1, static_cast<long long>(a.T - 1))] : h[0];
        const long long pn = g >= 2 ? h[min(g - 2, static_cast<long long>(a.T - 1))] : ls;
        const bool fts = g == 0, lts = ls >= a.tsb, pts = pn >= a.tsb;
        const int flags = (fts ? 1 : 0) | ((!fts && lts && pts) ? 2 : 0) | ((!fts && lts && !pts) ? 4 : 0) |
                          ((!fts && !lts && at >= 0) ? 8 : 0) | ((!fts && !lts) ? 16 : 0);
        ts_state[0] = ls;
        ts_state[1] = at >= 0 ? h[at] : h[0];
        ts_state[2] = flags;
        ts_state[3] = *a.max_initial;
      }
    }
    __syncthreads();
    last = ts_state[0];
    latest = ts_state[1];
    const int flags = static_cast<int>(ts_state[2]);
    first_ts = flags & 1;
    both = flags & 2;
    pair = flags & 4;
    fresh = flags & 8;
    check = (flags & 4) || (flags & 16);
    max_init = ts_state[3];
  }
  auto masked = [&](int v, bool su, bool be) {
    bool m = su || (first && be);
    if (TS) {
      const bool ts = v >= a.tsb;
      m = m || v == a.nots;
      m = m || (first_ts && (!ts || v > a.tsb + max_init));
      m = m || (both && ts);
      m = m || (pair && (v < a.eot || (ts && v < last)));
      m = m || (fresh && ts && v <= latest);
    }
    return m;
  };
  const float *x = a.logits + static_cast<size_t>(r) * V;
  // pass 1 (from HBM): online (max, sum of exponentials) of the raw logits, the masked ones and the masked
  // timestamps, the largest masked text logit; and each thread's best masked text / timestamp logit (its champions)
  Lse raw{-__builtin_huge_valf(), 0.f}, msk = raw, tss = raw;
  float mx_text = -__builtin_huge_valf();
  float ch_t = -__builtin_huge_valf(), ch_x = ch_t;  // champions: text (all tokens without timestamps), timestamps
  int ch_ti = kNoCand, ch_xi = kNoCand;
  const int tsb = TS ? a.tsb : V;  // (without timestamps every token counts as text)
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(a.suppress) & 1) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.begin) & 1) == 0;
  if constexpr (!TS) {
    // no timestamp rules: the masked maximum is the thread's champion (found per chunk, only when it grows), and
    // only a window's first row needs the raw sum (its no-speech probability)
    const bool want_raw = r == b * K;
    auto chunk = [&](const float (&xv)[kUnroll], const bool (&su)[kUnroll], const bool (&be)[kUnroll], int p0) {
      float xm[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) xm[u] = (su[u] || (first && be[u])) ? kLowest : xv[u];
      float cm = xm[0];
#pragma unroll
      for (int u = 1; u < kUnroll; ++u) cm = fmaxf(cm, xm[u]);
      if (cm > ch_t) {  // (rare after the first chunks) the first element equal to the chunk's maximum
        int at = kNoCand;
#pragma unroll
        for (int u = kUnroll - 1; u >= 0; --u)
          if (xm[u] == cm) at = chunk_v(p0, u);
        ch_t = cm;
        ch_ti = at;
      }
      lse_chunk<kUnroll>(msk, xm);
      if (want_raw) lse_chunk<kUnroll>(raw, xv);
    };
    int p0 = lo / 2;
    if (vec) {
      for (; 2 * (p0 + kScoreThreads * (kUnroll / 2)) <= hi; p0 += kScoreThreads * (kUnroll / 2)) {
        float xv[kUnroll];
        bool su[kUnroll], be[kUnroll];
        load_chunk<true, false>(x, a.suppress, a.begin, p0, hi, first, xv, su, be);
        chunk(xv, su, be, p0);
      }
    }
    for (; 2 * p0 < hi; p0 += kScoreThreads * (kUnroll / 2)) {
      float xv[kUnroll];
      bool su[kUnroll], be[kUnroll];
      load_chunk<false>(x, a.suppress, a.begin, p0, hi, first, xv, su, be);
      chunk(xv, su, be, p0);
    }
  } else {
    for (int p0 = lo / 2; 2 * p0 < hi; p0 += kScoreThreads * (kUnroll / 2)) {
      float xv[kUnroll], xm[kUnroll], xt[kUnroll];
      bool su[kUnroll], be[kUnroll];
      if (vec) load_chunk<true>(x, a.suppress, a.begin, p0, hi, first, xv, su, be);
      else load_chunk<false>(x, a.suppress, a.begin, p0, hi, first, xv, su, be);
  #pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int v = chunk_v(p0, u);
        xm[u] = v >= hi ? -__builtin_huge_valf() : (masked(v, su[u], be[u]) ? kLowest : xv[u]);
        if (TS) {
          xt[u] = v >= tsb ? xm[u] : -__builtin_huge_valf();
          if (v < tsb) {
            mx_text = fmaxf(mx_text, xm[u]);
            if (xm[u] > ch_t) {
              ch_t = xm[u];
              ch_ti = v;
            }
          } else if (xm[u] > ch_x) {
            ch_x = xm[u];
            ch_xi = v;
          }
        } else if (xm[u] > ch_t) {
          ch_t = xm[u];
          ch_ti = v;
        }
      }
      lse_chunk<kUnroll>(raw, xv);
      lse_chunk<kUnroll>(msk, xm);
      if (TS) lse_chunk<kUnroll>(tss, xt);
    }
  }
  raw = block_lse(raw, red);
  msk = block_lse(msk, red);
  if (TS) {
    tss = block_lse(tss, red);
    mx_text = block_reduce(mx_text, red, true);
  }
  if (tid == 0) {
    ex.red[0] = raw.m;
    ex.red[1] = raw.s;
    ex.red[2] = msk.m;
    ex.red[3] = msk.s;
    ex.red[4] = tss.m;
    ex.red[5] = tss.s;
    ex.red[6] = mx_text;
  }
  cluster.sync();
#pragma unroll
  for (int q = 0; q < kScoreCluster; ++q) {
    if (q == rank) continue;
    const Exchange<KK> *o = cluster.map_shared_rank(&ex, q);
    raw = lse_merge(raw, Lse{o->red[0], o->red[1]});
    msk = lse_merge(msk, Lse{o->red[2], o->red[3]});
    tss = lse_merge(tss, Lse{o->red[4], o->red[5]});
    mx_text = fmaxf(mx_text, o->red[6]);
  }
  const float m_raw = raw.m, s_raw = raw.s;
  float log_sum = logf(msk.s), base = msk.m;
  bool text_out = false;
  if (TS && check && tss.m > -__builtin_huge_valf()) {
    // text only if some text token is likelier than all timestamps together (search.py:335-338)
    const float lse = msk.m + log_sum;
    text_out = (tss.m - lse) + logf(tss.s) > mx_text - lse;
    if (text_out) {
      base = tss.m;
      log_sum = logf(tss.s);
    }
  }
  const float c = (a.sampling != nullptr && a.sampling[b] != 0) ? 0.f : a.cum[r];
  const int cand0 = (r - b * K) * V;
  if (r == b * K && rank == 0 && tid == 0) a.ns[b] = expf(x[a.no_speech] - (m_raw + logf(s_raw)));

  // The threshold: the kk-th best of the cluster's warp maxima of the threads' champions, in (masked logit, index)
  // order. The scores are a non-decreasing function of the masked logit, so every one of the row's best kk is at
  // least as good, or -- where two logits round to one score -- a few ulps below it; the candidates come from the
  // kk warps whose maxima are at least as good (few for any spread of values; a buffer overflow takes the exact
  // path).
  float ch_s;
  int ch_i;
  if (text_out) {  // the text tokens are now all masked: the thread's first text element stands for them
    const int v0 = lo + 2 * tid;  // (the thread's first element)
    const bool has_text = v0 < min(hi, tsb);
    ch_s = has_text ? kLowest : -__builtin_huge_valf();
    ch_i = has_text ? v0 : kNoCand;
  } else {
    ch_s = ch_t;
    ch_i = ch_ti;
  }
  if (better(ch_x, ch_xi, ch_s, ch_i)) {
    ch_s = ch_x;
    ch_i = ch_xi;
  }
  float wm_s = ch_s;
  int wm_i = ch_i;
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float s2 = __shfl_xor_sync(0xffffffffu, wm_s, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, wm_i, o);
    if (better(s2, i2, wm_s, wm_i)) {
      wm_s = s2;
      wm_i = i2;
    }
  }
  if (lane == 0) {
    ex.wm_s[warp] = wm_s;
    ex.wm_i[warp] = wm_i;
  }
  cluster.sync();
  __shared__ float thr_sh;
  __shared__ int thr_ish;
  if (warp == 0) {  // lane q: warp q % 8 of CTA q / 8; its rank among the 32 by counting
    static_assert(kScoreCluster * kScoreWarps == 32, "one warp ranks the cluster's warp maxima");
    const Exchange<KK> *o = cluster.map_shared_rank(&ex, lane / kScoreWarps);
    const float ms = o->wm_s[lane % kScoreWarps];
    const int mi = o->wm_i[lane % kScoreWarps];
    int rk = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) rk += better(__shfl_sync(0xffffffffu, ms, j), __shfl_sync(0xffffffffu, mi, j), ms, mi);
    const unsigned hit = __ballot_sync(0xffffffffu, rk == a.kk - 1);
    const int src_lane = hit ? __ffs(hit) - 1 : 31;  // (no kk-th: fewer finite values -- the last one)
    const float ts = __shfl_sync(0xffffffffu, ms, src_lane);
    const int ti = __shfl_sync(0xffffffffu, mi, src_lane);
    if (lane == 0) {
      thr_sh = hit ? ts : -__builtin_huge_valf();
      thr_ish = hit ? ti : kNoCand;
    }
  }
  __syncthreads();
  if (thr_sh <= kLowest) {
    // fewer than kk warps hold an unmasked logit (a window's first step with timestamps, or text masked in favour
    // of timestamps): the threshold from the threads' champions instead, exact -- the kk-th best of the cluster's
    float l1s[KK];
    int l1i[KK];
#pragma unroll
    for (int j = 0; j < KK; ++j) {
      l1s[j] = j == 0 ? ch_s : -__builtin_huge_valf();
      l1i[j] = j == 0 ? ch_i : kNoCand;
    }
    float ws[KK];
    int wi[KK];
    warp_select<KK>(l1s, l1i, a.kk, ws, wi);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < KK; ++j) {
        wl_s[warp][j] = j < a.kk ? ws[j] : -__builtin_huge_valf();
        wl_i[warp][j] = j < a.kk ? wi[j] : kNoCand;
      }
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < KK; ++j) {
        l1s[j] = lane < kScoreWarps ? wl_s[lane][j] : -__builtin_huge_valf();
        l1i[j] = lane < kScoreWarps ? wl_i[lane][j] : kNoCand;
      }
      warp_select<KK>(l1s, l1i, a.kk, ws, wi);
      if (lane == 0) {
#pragma unroll
        for (int j = 0; j < KK; ++j) {
          ex.ls[j] = j < a.kk ? ws[j] : -__builtin_huge_valf();
          ex.li[j] = j < a.kk ? wi[j] : kNoCand;
        }
      }
    }
    cluster.sync();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < KK; ++j) {
        const bool have = lane < kScoreCluster;
        const Exchange<KK> *o = cluster.map_shared_rank(&ex, have ? lane : 0);
        l1s[j] = have ? o->ls[j] : -__builtin_huge_valf();
        l1i[j] = have ? o->li[j] : kNoCand;
      }
      warp_select<KK>(l1s, l1i, a.kk, ws, wi);
      if (lane == 0) {
        float ts = ws[0];
        int ti = wi[0];
#pragma unroll
        for (int j = 1; j < KK; ++j)
          if (j == a.kk - 1) {
            ts = ws[j];
            ti = wi[j];
          }
        thr_sh = ts;
        thr_ish = ti;
      }
    }
    __syncthreads();
  }
  const float thr = thr_sh;
  const int thr_i = thr_ish;
  // rounding band below the threshold: a few ulps of the score computation's magnitudes
  const float band = (fabsf(thr) + fabsf(base) + fabsf(log_sum) + fabsf(c)) * 9.5367431640625e-7f;  // 2^-20
  const float thr_lo = thr - band;
  const bool all_lost = c == -__builtin_huge_valf();  // (every score -inf: the order is the index order)
  // pass 2 (from L2): the scores (written out if asked for) and the candidates, into shared memory
  float *out = a.scores ? a.scores + static_cast<size_t>(r) * V : nullptr;
  const float cut = all_lost ? kLowest : thr_lo;  // (every element below it is no candidate)
  auto consider = [&](int v, float xm) {
    if (xm >= cut || all_lost) {
      const bool cand = all_lost ? v - lo < a.kk : !(xm == thr && v > thr_i);
      if (cand) {
        const int slot = atomicAdd(&n_cand, 1);
        if (slot < a.cap) {
          cand_s[slot] = (xm - base - log_sum) + c;
          cand_i[slot] = cand0 + v;
        }
      }
    }
  };
  if (out == nullptr && !all_lost && cut > kLowest) {
    // the scores are not wanted: the logits alone, and the flags only of the (few) logits above the cut
    for (int p0 = lo / 2; 2 * p0 < hi; p0 += kScoreThreads * (kUnroll / 2)) {
      float xv[kUnroll];
      if (vec) load_logits<true>(x, p0, hi, xv);
      else load_logits<false>(x, p0, hi, xv);
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (xv[u] >= cut) {  // (a masked logit counts as kLowest, below any cut here)
          const int v = chunk_v(p0, u);
          const bool mk = masked(v, __ldg(a.suppress + v) != 0, first && __ldg(a.begin + v) != 0) ||
                          (TS && text_out && v < tsb);
          consider(v, mk ? kLowest : xv[u]);
        }
      }
    }
  } else {
    for (int p0 = lo / 2; 2 * p0 < hi; p0 += kScoreThreads * (kUnroll / 2)) {
      float xv[kUnroll];
      bool su[kUnroll], be[kUnroll];
      if (vec) load_chunk<true>(x, a.suppress, a.begin, p0, hi, first, xv, su, be);
      else load_chunk<false>(x, a.suppress, a.begin, p0, hi, first, xv, su, be);
  #pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int v = chunk_v(p0, u);
        if (v >= hi) continue;
        const bool mk = masked(v, su[u], be[u]) || (TS && text_out && v < tsb);
        const float xm = mk ? kLowest : xv[u];
        if (out) out[v] = (xm - base - log_sum) + c;
        consider(v, xm);
      }
    }
  }
  __syncthreads();
  if (n_cand > a.cap) {
    // (only adversarial near-ties overflow the buffer: this CTA's best kk by a per-thread sweep instead, exact)
    float l1s[KK];
    int l1i[KK];
#pragma unroll
    for (int j = 0; j < KK; ++j) {
      l1s[j] = -__builtin_huge_valf();
      l1i[j] = kNoCand;
    }
    for (int v = lo + tid; v < hi; v += kScoreThreads) {
      const bool mk = masked(v, __ldg(a.suppress + v) != 0, __ldg(a.begin + v) != 0) || (TS && text_out && v < tsb);
      insert<KK>(l1s, l1i, ((mk ? kLowest : __ldg(x + v)) - base - log_sum) + c, cand0 + v);
    }
    float ws[KK];
    int wi[KK];
    warp_select<KK>(l1s, l1i, a.kk, ws, wi);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < KK; ++j) {
        wl_s[warp][j] = j < a.kk ? ws[j] : -__builtin_huge_valf();
        wl_i[warp][j] = j < a.kk ? wi[j] : kNoCand;
      }
    }
    __syncthreads();
    if (tid < kScoreWarps * a.kk) {  // every warp's list becomes a candidate
      cand_s[tid] = wl_s[tid / a.kk][tid % a.kk];
      cand_i[tid] = wl_i[tid / a.kk][tid % a.kk];
    }
    __syncthreads();
    if (tid == 0) n_cand = kScoreWarps * a.kk;
    __syncthreads();
  }
  // the row's best kk: rank 0 ranks the cluster's candidates directly when they are few (always, but for
  // adversarial near-ties); otherwise every CTA selects its best kk and rank 0 merges those (the exact path)
  if (tid == 0) ex.n_cand = n_cand;
  cluster.sync();
  int total = 0;
  bool few = true;
#pragma unroll
  for (int q = 0; q < kScoreCluster; ++q) {
    const int nq = cluster.map_shared_rank(&ex, q)->n_cand;
    few = few && nq <= a.cap;
    total += min(nq, a.cap);
  }
  few = few && total <= kGather;
  __shared__ float g_s[kGather];
  __shared__ int g_i[kGather];
  if (few) {
    if (rank == 0 && warp == 0) {
      int at = 0;
#pragma unroll
      for (int q = 0; q < kScoreCluster; ++q) {
        const int nq = cluster.map_shared_rank(&ex, q)->n_cand;
        const float *qs = cluster.map_shared_rank(cand_s, q);
        const int *qi = cluster.map_shared_rank(cand_i, q);
        for (int j = lane; j < nq; j += 32) {
          g_s[at + j] = qs[j];
          g_i[at + j] = qi[j];
        }
        at += nq;
      }
      __syncwarp();
      float *rs = a.row_s + static_cast<size_t>(r) * a.kk;
      int *ri = a.row_i + static_cast<size_t>(r) * a.kk;
      for (int j = lane; j < total; j += 32) {
        const float sj = g_s[j];
        const int ij = g_i[j];
        int rk = 0;
        for (int q = 0; q < total; ++q) rk += better(g_s[q], g_i[q], sj, ij);
        if (rk < a.kk) {
          rs[rk] = sj;
          ri[rk] = ij;
        }
      }
      for (int j = total + lane; j < a.kk; j += 32) {  // (fewer candidates than kk: tiny vocabularies)
        rs[j] = -__builtin_huge_valf();
        ri[j] = kNoCand;
      }
    }
  } else {
    if (warp == 0) {
      float l1s[KK];
      int l1i[KK];
  #pragma unroll
      for (int j = 0; j < KK; ++j) {
        l1s[j] = -__builtin_huge_valf();
        l1i[j] = kNoCand;
      }
      const int nc = min(n_cand, a.cap);
      for (int q = lane; q < nc; q += 32) insert<KK>(l1s, l1i, cand_s[q], cand_i[q]);
      float ws[KK];
      int wi[KK];
      warp_select<KK>(l1s, l1i, a.kk, ws, wi);
      if (lane == 0) {
  #pragma unroll
        for (int j = 0; j < KK; ++j) {
          ex.ls[j] = j < a.kk ? ws[j] : -__builtin_huge_valf();
          ex.li[j] = j < a.kk ? wi[j] : kNoCand;
        }
      }
    }
    cluster.sync();
    if (rank == 0 && warp == 0) {
      float l1s[KK];
      int l1i[KK];
  #pragma unroll
      for (int j = 0; j < KK; ++j) {
        const bool have = lane < kScoreCluster;
        const Exchange<KK> *o = cluster.map_shared_rank(&ex, have ? lane : 0);
        l1s[j] = have ? o->ls[j] : -__builtin_huge_valf();
        l1i[j] = have ? o->li[j] : kNoCand;
      }
      float ws[KK];
      int wi[KK];
      warp_select<KK>(l1s, l1i, a.kk, ws, wi);
      float *rs = a.row_s + static_cast<size_t>(r) * a.kk;
      int *ri = a.row_i + static_cast<size_t>(r) * a.kk;
      if (lane < a.kk) {
        float sv = ws[0];
        int iv = wi[0];
  #pragma unroll
        for (int j = 1; j < KK; ++j)
          if (lane == j) {
            sv = ws[j];
            iv = wi[j];
          }
        rs[lane] = sv;
        ri[lane] = iv;
      }
    }
  }
  cluster.sync();  // (no CTA leaves while rank 0 may still read its shared memory)
  if (rank != 0 || warp != 0) return;
  __threadfence();
  __syncwarp();
  if (lane == 0) is_last = atomicAdd(a.counters + b, 1) == K - 1;
  __syncwarp();
  if (!is_last) return;
  __threadfence();
  // the window's best kk over its K rows' lists (lane k < K holds row b*K + k's list)
  float l1s[KK];
  int l1i[KK];
#pragma unroll
  for (int j = 0; j < KK; ++j) {
    const bool have = lane < K && j < a.kk;
    l1s[j] = have ? __ldcg(a.row_s + static_cast<size_t>(b * K + lane) * a.kk + j) : -__builtin_huge_valf();
    l1i[j] = have ? __ldcg(a.row_i + static_cast<size_t>(b * K + lane) * a.kk + j) : kNoCand;
  }
  float ws[KK];
  int wi[KK];
  warp_select<KK>(l1s, l1i, a.kk, ws, wi);
  if (lane < a.kk) {
    float sv = ws[0];
    int iv = wi[0];
#pragma unroll
    for (int j = 1; j < KK; ++j)
      if (lane == j) {
        sv = ws[j];
        iv = wi[j];
      }
    a.top_s[static_cast<size_t>(b) * a.kk + lane] = sv;
    a.top_i[static_cast<size_t>(b) * a.kk + lane] = static_cast<int64_t>(iv);
  }
  if (lane == 0) a.counters[b] = 0;  // left zeroed for the next launch
}

template <int KK, bool TS>
int launch_scores(const ScoreArgs &a, int n, void *stream) {
  auto kernel = beam_scores_kernel<KK, TS>;
  const int smem = a.cap * static_cast<int>(sizeof(float) + sizeof(int));
  const int st = opt_in_smem<beam_scores_kernel<KK, TS>>(smem, "beam_scores");
  if (st != WT_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n * kScoreCluster);
  cfg.blockDim = dim3(kScoreThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[2];
  int na = 0;
  attr[na].id = cudaLaunchAttributeClusterDimension;
  attr[na].val.clusterDim.x = kScoreCluster;
  attr[na].val.clusterDim.y = 1;
  attr[na].val.clusterDim.z = 1;
  ++na;
  if (launch_flags() & WT_LAUNCH_PDL) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a);
  if (e != cudaSuccess) return fail(WT_ERR_CUDA, "beam_scores: %s", cudaGetErrorString(e));
  return WT_OK;
}

size_t scores_workspace(int windows, int beams) {
  const size_t n = static_cast<size_t>(windows) * beams, kk = 2 * static_cast<size_t>(beams);
  const size_t counters = (static_cast<size_t>(windows) * sizeof(int) + 255) / 256 * 256;
  const size_t lists_s = (n * kk * sizeof(float) + 255) / 256 * 256;
  return counters + lists_s + n * kk * sizeof(int);
}

}  // namespace
}  // namespace wt

extern "C" {

size_t wt_beam_scores_workspace(int windows, int beams) {
  if (windows <= 0 || beams <= 0) return 0;
  return wt::scores_workspace(windows, beams);
}

int wt_beam_scores(const float *logits, const uint8_t *suppress, const uint8_t *begin, const int64_t *t,
                   const float *cum, const int64_t *hist, const int64_t *max_initial, float *scores, float *ns,
                   float *top_s, int64_t *top_i, int windows, int beams, int vocab, int hist_len, int timestamps,
                   int no_speech, int no_timestamps, int ts_begin, int eot, void *workspace, size_t workspace_bytes,
                   void *stream) {
  return wt_beam_scores_mixed(logits, suppress, begin, t, cum, nullptr, hist, max_initial, scores, ns, top_s, top_i,
                              windows, beams, vocab, hist_len, timestamps, no_speech, no_timestamps, ts_begin, eot,
                              workspace, workspace_bytes, stream);
}

int wt_beam_scores_mixed(const float *logits, const uint8_t *suppress, const uint8_t *begin, const int64_t *t,
                         const float *cum, const uint8_t *sampling, const int64_t *hist, const int64_t *max_initial,
                         float *scores, float *ns, float *top_s, int64_t *top_i, int windows, int beams, int vocab,
                         int hist_len, int timestamps, int no_speech, int no_timestamps, int ts_begin, int eot,
                         void *workspace, size_t workspace_bytes, void *stream) {
  using namespace wt;
  WT_REQUIRE(windows > 0 && beams > 0 && vocab > 0 && hist_len > 0, WT_ERR_ARG,
             "beam_scores: sizes must be positive (windows %d, beams %d, vocab %d, hist_len %d)", windows, beams,
             vocab, hist_len);
  WT_REQUIRE(logits && suppress && begin && t && cum && hist && max_initial && ns && top_s && top_i, WT_ERR_ARG,
             "beam_scores: null pointer");
  WT_REQUIRE(static_cast<long long>(beams) * vocab < (1LL << 31) - 1 &&
                 static_cast<long long>(windows) * beams < (1LL << 31),
             WT_ERR_ARG, "beam_scores: too large");
  WT_REQUIRE(no_speech >= 0 && no_speech < vocab && eot >= 0 && eot < vocab, WT_ERR_ARG,
             "beam_scores: token ids outside the vocabulary");
  WT_REQUIRE(!timestamps || (ts_begin > 0 && ts_begin < vocab && no_timestamps >= 0 && no_timestamps < vocab),
             WT_ERR_ARG, "beam_scores: timestamps need ts_begin and no_timestamps inside the vocabulary");
  const size_t need = scores_workspace(windows, beams);
  WT_REQUIRE(workspace && workspace_bytes >= need, WT_ERR_WORKSPACE,
             "beam_scores: needs a zeroed workspace of %zu bytes (given %zu)", need, workspace ? workspace_bytes : 0);
  WT_ALIGNED(workspace);
  const int n = windows * beams, kk = 2 * beams;
  char *ws = static_cast<char *>(workspace);
  const size_t counters = (static_cast<size_t>(windows) * sizeof(int) + 255) / 256 * 256;
  const size_t lists_s = (static_cast<size_t>(n) * kk * sizeof(float) + 255) / 256 * 256;
  // candidate buffer per CTA: kk threads' worth of elements (see the kernel's threshold)
  const int per_cta = (vocab + kScoreCluster - 1) / kScoreCluster;
  const int cap = kk * max(kScoreWarps, (per_cta + kScoreThreads - 1) / kScoreThreads) + 64;
  WT_REQUIRE(cap * 8 <= 160 * 1024, WT_ERR_UNSUPPORTED, "beam_scores: vocabulary %d too large", vocab);
  ScoreArgs a{logits, suppress, begin, t, hist, max_initial, cum, sampling, scores, ns, top_s, top_i,
              reinterpret_cast<float *>(ws + counters), reinterpret_cast<int *>(ws + counters + lists_s),
              reinterpret_cast<int *>(ws), beams, vocab, hist_len, kk, cap, timestamps, no_speech, no_timestamps,
              ts_begin, eot};
  if (timestamps) {
    if (kk <= 4) return launch_scores<4, true>(a, n, stream);
    if (kk <= 8) return launch_scores<8, true>(a, n, stream);
    if (kk <= 12) return launch_scores<12, true>(a, n, stream);
    if (kk <= 16) return launch_scores<16, true>(a, n, stream);
  } else {
    if (kk <= 4) return launch_scores<4, false>(a, n, stream);
    if (kk <= 8) return launch_scores<8, false>(a, n, stream);
    if (kk <= 12) return launch_scores<12, false>(a, n, stream);
    if (kk <= 16) return launch_scores<16, false>(a, n, stream);
  }
  return fail(WT_ERR_UNSUPPORTED, "beam_scores: %d beams (supported: up to 8)", beams);
}

}  // extern "C"
