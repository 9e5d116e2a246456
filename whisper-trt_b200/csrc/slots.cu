// KV-cache append / gather and the slot-table bookkeeping of beam search (integer work, bit-exact).
//
// Beam search never moves the KV cache: row r's table src[r, :] names, per cache slot, the row whose cache holds
// it (reference search.py:1-26 docstring, :242-265, :367-409; fused beam_kernels.py:169-269). These kernels are
// HBM-light (a few hundred KB a step) and latency-bound; they are written so that one step needs one launch:
//   * one CTA per window; the window's rows read each other's rows (a new beam takes its parent's table), so each
//     THREAD owns whole columns: it reads column cc of every parent row and writes column cc of every new row,
//     no other thread touches that column -- no shared-memory copy and no barrier between reads and writes;
//   * the per-window scalar rules (CTranslate2's candidate selection) run once per window in shared memory.
#include "common.cuh"

namespace wt {
namespace {

constexpr int kMaxBeams = 32;

// ---- append / gather ------------------------------------------------------------------------------------
template <int CHUNKS>  // 16-byte chunks per (row, head) = D * 2 / 16
__global__ void cache_append_kernel(const uint4 *__restrict__ qkv, uint4 *kc, uint4 *vc,
                                    const int64_t *__restrict__ offset, int N, int H, int C) {
  pdl_wait();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long long>(N) * H * CHUNKS) return;
  const int ch = static_cast<int>(i % CHUNKS);
  const long long rh = i / CHUNKS;
  const int r = static_cast<int>(rh / H), h = static_cast<int>(rh % H);
  const int64_t o = offset[r];
  if (o < 0 || o >= C) return;
  const size_t hd = static_cast<size_t>(H) * CHUNKS;
  const size_t srcq = static_cast<size_t>(r) * 3 * hd + static_cast<size_t>(h) * CHUNKS + ch;
  const size_t dst = ((static_cast<size_t>(r) * H + h) * C + o) * CHUNKS + ch;
  kc[dst] = qkv[srcq + hd];
  vc[dst] = qkv[srcq + 2 * hd];
}

__global__ void gather_cache_kernel(const uint4 *__restrict__ cache, const int32_t *__restrict__ src,
                                    uint4 *__restrict__ out, int N, int H, int C, int chunks) {
  pdl_wait();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(N) * H * C * chunks;
  if (i >= total) return;
  const int ch = static_cast<int>(i % chunks);
  long long t = i / chunks;
  const int j = static_cast<int>(t % C);
  t /= C;
  const int h = static_cast<int>(t % H);
  const int r = static_cast<int>(t / H);
  int row = src[static_cast<size_t>(r) * C + j];
  row = row < 0 ? 0 : (row > N - 1 ? N - 1 : row);
  out[i] = cache[((static_cast<size_t>(row) * H + h) * C + j) * chunks + ch];
}

// ---- beam reorder: parents given ---------------------------------------------------------------------------
template <int KMAX>
__global__ void __launch_bounds__(128)
    beam_reorder_kernel(int32_t *src, int64_t *hist, const int64_t *__restrict__ token,
                        const int64_t *__restrict__ t, const int64_t *__restrict__ parent, int64_t *pos,
                        const uint8_t *__restrict__ live, int64_t *offset, int K, int C, int T, int advance) {
  const int b = blockIdx.x;
  pdl_wait();
  const bool is_live = live == nullptr || live[b] != 0;
  const int64_t pb = pos[b];
  if (is_live) {
    int par[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k) {
      int64_t p = k < K ? parent[b * K + k] : 0;
      p = p < 0 ? 0 : (p > K - 1 ? K - 1 : p);  // (clamped: a bad parent index never reads another window)
      par[k] = b * K + static_cast<int>(p);
    }
    for (int cc = threadIdx.x; cc < C; cc += blockDim.x) {
      int32_t vals[KMAX];
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (k < K) vals[k] = src[static_cast<size_t>(par[k]) * C + cc];
#pragma unroll
      for (int k = 0; k < KMAX; ++k)
        if (k < K) src[static_cast<size_t>(b * K + k) * C + cc] = (cc == pb) ? par[k] : vals[k];
    }
    if (hist != nullptr) {
      const int64_t tb = t != nullptr ? t[b] : -1;
      for (int tt = threadIdx.x; tt < T; tt += blockDim.x) {
        int64_t vals[KMAX];
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
          if (k < K) vals[k] = hist[static_cast<size_t>(par[k]) * T + tt];
#pragma unroll
        for (int k = 0; k < KMAX; ++k)
          if (k < K)
            hist[static_cast<size_t>(b * K + k) * T + tt] =
                (token != nullptr && tt == tb) ? token[b * K + k] : vals[k];
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && is_live && advance) pos[b] = pb + 1;
  if (offset != nullptr && threadIdx.x < K) offset[b * K + threadIdx.x] = (is_live && advance) ? pb + 1 : pb;
}

// ---- beam update: CTranslate2's rules from the best 2K candidates (beam_kernels.py:169-269, beam mode) --------
struct UpdateArgs {
  const float *top_s;
  const int64_t *top_i;
  int64_t *t, *pos;
  const int64_t *sot_pos;
  const float *ns;
  float *no_speech;
  uint8_t *done;
  int64_t *hist;
  float *cum;
  int32_t *src;
  int64_t *tokens;
  const int64_t *forced;
  int64_t *h_count;
  float *h_score;
  int64_t *h_len, *h_tokens;
  const int64_t *last_t;
  // sampled slots (all null when the search has none, as wt_beam_update passes): per window whether it is sampled,
  // per row its sampled token and that token's log-probability (wt_beam_sample), whether it is done, its length
  const uint8_t *sampling;
  const int64_t *samp_tok;
  const float *samp_score;
  uint8_t *row_done;
  int64_t *length;
  int K, C, T, S, P, V, eot;
};

__device__ __forceinline__ int clamp_beam(int64_t p, int K) {
  return static_cast<int>(p < 0 ? 0 : (p > K - 1 ? K - 1 : p));  // (a bad candidate never reads another window)
}

template <int KMAX>
__global__ void __launch_bounds__(128) beam_update_kernel(UpdateArgs a) {
  const int b = blockIdx.x, tid = threadIdx.x;
  const int K = a.K, C = a.C, T = a.T;
  __shared__ int s_mode;  // 0: untouched, 1: prompt token, 2: beam step, 3: sampled step
  __shared__ int64_t s_tb, s_pb;
  __shared__ int s_live_rows;
  __shared__ int s_par[KMAX], s_newpar[KMAX], s_slot[KMAX];
  __shared__ int64_t s_tok[KMAX], s_newtok[KMAX];
  __shared__ float s_ps[KMAX], s_news[KMAX];
  __shared__ uint8_t s_finish[KMAX], s_eos[KMAX];
  __shared__ int s_ended;
  pdl_wait();
  if (tid == 0) {
    const int64_t tb = a.t[b], pb = a.pos[b];
    const bool db = a.done[b] != 0;
    s_tb = tb;
    s_pb = pb;
    if (pb == a.sot_pos[b]) a.no_speech[b] = a.ns[b];
    const bool sampled = a.sampling != nullptr && a.sampling[b] != 0;
    s_mode = tb < 0 ? 1 : (db ? 0 : (sampled ? 3 : 2));
    s_live_rows = 0;
    if (s_mode == 2) {
      const int64_t *ti = a.top_i + static_cast<size_t>(b) * 2 * K;
      const float *ts = a.top_s + static_cast<size_t>(b) * 2 * K;
      const bool last = tb == a.last_t[b];
      int64_t count = a.h_count[b];
      int n_fin = 0, n_eos = 0, n_sec_ok = 0;
      for (int k = 0; k < K; ++k) n_sec_ok += (ti[K + k] % a.V) != a.eot;
      for (int k = 0; k < K; ++k) {
        const int64_t tok = ti[k] % a.V;
        const int par = clamp_beam(ti[k] / a.V, K);
        const bool eos = tok == a.eot;
        const bool fin = eos || last;
        s_tok[k] = tok;
        s_par[k] = par;
        s_ps[k] = ts[k];
        s_eos[k] = eos;
        s_finish[k] = fin;
        s_slot[k] = static_cast<int>(count + n_fin);  // h_count + cumsum(finish) - 1 (for finished ones)
        n_fin += fin;
        // an ended candidate takes the r-th secondary candidate that does not end (r = its rank among the ended)
        int64_t nt = tok;
        int np = par;
        float nsc = ts[k];
        if (eos) {
          const int r = n_eos++;
          if (r < n_sec_ok) {
            int seen = 0;
            for (int j = 0; j < K; ++j) {
              const int64_t st = ti[K + j] % a.V;
              if (st != a.eot) {
                if (seen == r) {
                  nt = st;
                  np = clamp_beam(ti[K + j] / a.V, K);
                  nsc = ts[K + j];
                  break;
                }
                ++seen;
              }
            }
          }
        }
        s_newtok[k] = nt;
        s_newpar[k] = np;
        s_news[k] = nsc;
      }
      count += n_fin;
      s_ended = (count >= K) || last;
      a.h_count[b] = count;
    }
  }
  __syncthreads();
  const int mode = s_mode;
  if (mode == 0) return;
  const int64_t tb = s_tb, pb = s_pb;
  if (mode == 1) {  // in the prompt: its next token, the rows mark their new slot (beam_kernels.py:186-192)
    if (tid < K) {
      const int r = b * K + tid;
      const int P = a.P;
      int64_t idx = (P + tb) < P ? (P + tb) : P;
      idx = idx < 0 ? 0 : idx;
      a.tokens[r] = a.forced[static_cast<size_t>(b) * (P + 1) + idx];
      if (pb >= 0 && pb < C) a.src[static_cast<size_t>(r) * C + pb] = r;
    }
    __syncthreads();
    if (tid == 0) {
      a.pos[b] = pb + 1;
      a.t[b] = tb + 1;
    }
    return;
  }
  if (mode == 3) {  // a sampled window: GreedySearch's rules on each row's own sampled token (beam_kernels.py:200-225)
    if (tid < K) {
      const int r = b * K + tid;
      const int64_t tok = a.samp_tok[r];
      bool rd = a.row_done[r] != 0;
      if (!rd) a.cum[r] = a.cum[r] + a.samp_score[r];
      const bool eos = tok == a.eot, last = tb == a.last_t[b];
      if (!rd && !eos) {  // a generated token (EOS is not part of the hypothesis)
        if (tb >= 0 && tb < T) a.hist[static_cast<size_t>(r) * T + tb] = tok;
        a.length[r] += 1;
      }
      rd = rd || eos || last;
      a.row_done[r] = rd;
      a.tokens[r] = tok;
      if (pb >= 0 && pb < C) a.src[static_cast<size_t>(r) * C + pb] = r;  // the row's own new slot
      if (!rd) atomicAdd(&s_live_rows, 1);
    }
    __syncthreads();
    if (tid == 0) {
      const bool ended = s_live_rows == 0;
      a.done[b] = ended;
      if (!ended) {
        a.pos[b] = pb + 1;
        a.t[b] = tb + 1;
      }
    }
    return;
  }
  // beam step: every read of the window's rows before any write, column by column per thread
  for (int cc = tid; cc < C; cc += blockDim.x) {
    int32_t vals[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) vals[k] = a.src[static_cast<size_t>(b * K + s_newpar[k]) * C + cc];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) a.src[static_cast<size_t>(b * K + k) * C + cc] = (cc == pb) ? b * K + s_newpar[k] : vals[k];
  }
  for (int tt = tid; tt < T; tt += blockDim.x) {
    int64_t ph[KMAX], nh[KMAX];
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) {
        ph[k] = a.hist[static_cast<size_t>(b * K + s_par[k]) * T + tt];
        nh[k] = a.hist[static_cast<size_t>(b * K + s_newpar[k]) * T + tt];
      }
#pragma unroll
    for (int k = 0; k < KMAX; ++k)
      if (k < K) {
        if (s_finish[k] && static_cast<unsigned>(s_slot[k]) < static_cast<unsigned>(a.S))  // finished hypothesis: EOS not part of it; at the last step the token is
          a.h_tokens[(static_cast<size_t>(b) * a.S + s_slot[k]) * T + tt] =
              (!s_eos[k] && tt == tb) ? s_tok[k] : ph[k];
        a.hist[static_cast<size_t>(b * K + k) * T + tt] = (tt == tb) ? s_newtok[k] : nh[k];
      }
  }
  if (tid < K && s_finish[tid] && static_cast<unsigned>(s_slot[tid]) < static_cast<unsigned>(a.S)) {
    a.h_score[static_cast<size_t>(b) * a.S + s_slot[tid]] = s_ps[tid];
    a.h_len[static_cast<size_t>(b) * a.S + s_slot[tid]] = tb + (s_eos[tid] ? 0 : 1);
  }
  if (tid < K) {
    const int r = b * K + tid;
    a.cum[r] = s_news[tid];
    a.tokens[r] = s_newtok[tid];
  }
  __syncthreads();
  if (tid == 0) {
    a.done[b] = s_ended;
    if (!s_ended) {
      a.pos[b] = pb + 1;
      a.t[b] = tb + 1;
    }
  }
}

// ---- sampled slots: each sampled row's token by Gumbel-max (beam_kernels.py:136-167; search.py:104-129,342-346) -----
// The reference's counter-based uniform (search.uniform): a 32-bit counter of (seed, step, row within the window,
// token) through PCG's output permutation twice, in 64-bit integer arithmetic masked to 32 bits, then
// (float(x) + 0.5) / 2^32 -- a function of the window's seed and step only, so a window draws the same numbers in any
// slot and inside a CUDA graph (no generator state).
__device__ __forceinline__ float counter_uniform(int64_t x) {
  constexpr uint64_t m = 0xFFFFFFFFull;
  uint64_t v = static_cast<uint64_t>(x) & m;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    v = (v * 747796405ull + 2891336453ull) & m;
    v = (((v >> ((v >> 28) + 4)) ^ v) * 277803737ull) & m;
    v = ((v >> 22) ^ v) & m;
  }
  return (__ull2float_rn(v) + 0.5f) * (1.0f / 4294967296.0f);
}

struct SampleArgs {
  const float *scores;  // [N, V]: log-probabilities of the sampled rows (wt_beam_scores_mixed)
  const int64_t *t;
  const uint8_t *done, *row_done, *sampling;
  const float *temperature;
  const int64_t *seed;
  int64_t *samp_tok;
  float *samp_score;
  int K, V;
};

constexpr int kSampleThreads = 256;

// One CTA per row: g = score / temperature - log(-log(max(u, 1e-20))) over the vocabulary, its first maximum.
__global__ void __launch_bounds__(kSampleThreads) beam_sample_kernel(SampleArgs a) {
  const int r = blockIdx.x, b = r / a.K, tid = threadIdx.x;
  pdl_wait();
  pdl_launch_dependents();
  const int64_t tw = a.t[b];
  if (!(a.sampling[b] != 0 && a.done[b] == 0 && tw >= 0 && a.row_done[r] == 0)) return;  // (the whole CTA)
  const float temp = a.temperature[b];
  const int64_t mix = a.seed[b] * 0x6C8E9CF5LL + tw * 0x85EBCA77LL + static_cast<int64_t>(r % a.K) * a.V;
  const float *x = a.scores + static_cast<size_t>(r) * a.V;
  float best = kNegInf;
  int bi = a.V;
  for (int v = tid; v < a.V; v += kSampleThreads) {  // (ascending per thread: a strict > keeps the first maximum)
    const float u = fmaxf(counter_uniform(mix + v), 1e-20f);
    const float g = __fdiv_rn(x[v], temp) - logf(-logf(u));
    if (g > best) {
      best = g;
      bi = v;
    }
  }
  __shared__ float s_best[kSampleThreads / 32];
  __shared__ int s_bi[kSampleThreads / 32];
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ob > best || (ob == best && oi < bi)) {
      best = ob;
      bi = oi;
    }
  }
  if ((tid & 31) == 0) {
    s_best[tid >> 5] = best;
    s_bi[tid >> 5] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kSampleThreads / 32; ++w)
      if (s_best[w] > best || (s_best[w] == best && s_bi[w] < bi)) {
        best = s_best[w];
        bi = s_bi[w];
      }
    if (bi >= a.V) bi = 0;  // (no candidate compared greater than -inf: the reference keeps index 0)
    a.samp_tok[r] = bi;
    a.samp_score[r] = x[bi];
  }
}

__global__ void slot_reset_kernel(int32_t *src, const int64_t *__restrict__ slots, int W, int K, int C,
                                  int prefilled) {
  pdl_wait();
  const int i = blockIdx.x;  // slot index in `slots`
  const int64_t s = slots[i];
  if (s < 0 || s >= W) return;  // (slots outside [0, windows) are ignored)
  for (int e = threadIdx.x; e < K * C; e += blockDim.x) {
    const int k = e / C, cc = e - k * C;
    const int64_t r = s * K + k;
    src[static_cast<size_t>(r) * C + cc] = static_cast<int32_t>(prefilled ? s * K : r);
  }
}

}  // namespace
}  // namespace wt

extern "C" {

int wt_cache_append(int dtype, const void *qkv, void *k_cache, void *v_cache, const int64_t *offset, int rows,
                    int heads, int capacity, int head_dim, void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && heads > 0 && capacity > 0 && head_dim > 0, WT_ERR_ARG, "cache_append: sizes must be positive");
  WT_REQUIRE(qkv && k_cache && v_cache && offset, WT_ERR_ARG, "cache_append: null pointer");
  WT_REQUIRE(dtype == WT_F16 || dtype == WT_BF16, WT_ERR_DTYPE, "cache_append: unknown dtype %d", dtype);
  WT_ALIGNED(qkv);
  WT_ALIGNED(k_cache);
  WT_ALIGNED(v_cache);
  WT_ALIGNED(offset);
  const long long total = static_cast<long long>(rows) * heads * (head_dim / 8);
  const dim3 grid(static_cast<unsigned>((total + 255) / 256)), block(256);
  auto *q = static_cast<const uint4 *>(qkv);
  auto *kc = static_cast<uint4 *>(k_cache);
  auto *vc = static_cast<uint4 *>(v_cache);
  switch (head_dim) {
    case 16: return launch("cache_append", cache_append_kernel<2>, grid, block, 0, stream, q, kc, vc, offset, rows, heads, capacity);
    case 32: return launch("cache_append", cache_append_kernel<4>, grid, block, 0, stream, q, kc, vc, offset, rows, heads, capacity);
    case 64: return launch("cache_append", cache_append_kernel<8>, grid, block, 0, stream, q, kc, vc, offset, rows, heads, capacity);
    case 128: return launch("cache_append", cache_append_kernel<16>, grid, block, 0, stream, q, kc, vc, offset, rows, heads, capacity);
    default: return fail(WT_ERR_UNSUPPORTED, "cache_append: head_dim %d (supported: 16, 32, 64, 128)", head_dim);
  }
}

int wt_gather_cache(int dtype, const void *cache, const int32_t *src, void *out, int rows, int heads,
                    int capacity, int head_dim, void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && heads > 0 && capacity > 0 && head_dim > 0, WT_ERR_ARG, "gather_cache: sizes must be positive");
  WT_REQUIRE(cache && src && out, WT_ERR_ARG, "gather_cache: null pointer");
  WT_REQUIRE(dtype == WT_F16 || dtype == WT_BF16, WT_ERR_DTYPE, "gather_cache: unknown dtype %d", dtype);
  WT_REQUIRE(head_dim % 8 == 0, WT_ERR_UNSUPPORTED, "gather_cache: head_dim %d not a multiple of 8", head_dim);
  WT_ALIGNED(cache);
  WT_ALIGNED(src);
  WT_ALIGNED(out);
  const int chunks = head_dim / 8;
  const long long total = static_cast<long long>(rows) * heads * capacity * chunks;
  WT_REQUIRE(total < (1LL << 31) * 256, WT_ERR_ARG, "gather_cache: too large");
  return launch("gather_cache", gather_cache_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256),
                0, stream, static_cast<const uint4 *>(cache), src, static_cast<uint4 *>(out), rows, heads,
                capacity, chunks);
}

int wt_beam_reorder(int32_t *src, int64_t *hist, const int64_t *token, const int64_t *t, const int64_t *parent,
                    int64_t *pos, const uint8_t *live, int64_t *offset, int windows, int beams, int capacity,
                    int hist_len, int advance, void *stream) {
  using namespace wt;
  WT_REQUIRE(windows > 0 && beams > 0 && capacity > 0, WT_ERR_ARG, "beam_reorder: sizes must be positive");
  WT_REQUIRE(beams <= kMaxBeams, WT_ERR_UNSUPPORTED, "beam_reorder: at most %d beams", kMaxBeams);
  WT_REQUIRE(src && parent && pos, WT_ERR_ARG, "beam_reorder: null pointer");
  WT_REQUIRE(hist == nullptr || hist_len > 0, WT_ERR_ARG, "beam_reorder: hist_len must be positive");
  WT_REQUIRE(token == nullptr || (hist != nullptr && t != nullptr), WT_ERR_ARG,
             "beam_reorder: token needs hist and t");
  const dim3 grid(windows), block(128);
  if (beams <= 8)
    return launch("beam_reorder", beam_reorder_kernel<8>, grid, block, 0, stream, src, hist, token, t, parent, pos,
                  live, offset, beams, capacity, hist_len, advance);
  return launch("beam_reorder", beam_reorder_kernel<32>, grid, block, 0, stream, src, hist, token, t, parent, pos,
                live, offset, beams, capacity, hist_len, advance);
}

int wt_beam_update(const float *top_s, const int64_t *top_i, int64_t *t, int64_t *pos, const int64_t *sot_pos,
                   const float *ns, float *no_speech, uint8_t *done, int64_t *hist, float *cum, int32_t *src,
                   int64_t *tokens, const int64_t *forced, int64_t *h_count, float *h_score, int64_t *h_len,
                   int64_t *h_tokens, const int64_t *last_t, int windows, int beams, int capacity, int hist_len,
                   int hyp_slots, int prompt_len, int vocab, int eot, void *stream) {
  return wt_beam_update_mixed(top_s, top_i, t, pos, sot_pos, ns, no_speech, done, hist, cum, src, tokens, forced,
                              h_count, h_score, h_len, h_tokens, last_t, nullptr, nullptr, nullptr, nullptr, nullptr,
                              windows, beams, capacity, hist_len, hyp_slots, prompt_len, vocab, eot, stream);
}

int wt_beam_update_mixed(const float *top_s, const int64_t *top_i, int64_t *t, int64_t *pos, const int64_t *sot_pos,
                         const float *ns, float *no_speech, uint8_t *done, int64_t *hist, float *cum, int32_t *src,
                         int64_t *tokens, const int64_t *forced, int64_t *h_count, float *h_score, int64_t *h_len,
                         int64_t *h_tokens, const int64_t *last_t, const uint8_t *sampling, const int64_t *samp_tok,
                         const float *samp_score, uint8_t *row_done, int64_t *length, int windows, int beams,
                         int capacity, int hist_len, int hyp_slots, int prompt_len, int vocab, int eot,
                         void *stream) {
  using namespace wt;
  WT_REQUIRE(sampling == nullptr || (samp_tok && samp_score && row_done && length), WT_ERR_ARG,
             "beam_update: sampled slots need samp_tok, samp_score, row_done and length");
  WT_REQUIRE(windows > 0 && beams > 0 && capacity > 0 && hist_len > 0 && vocab > 0 && prompt_len >= 1, WT_ERR_ARG,
             "beam_update: sizes must be positive");
  WT_REQUIRE(beams <= kMaxBeams, WT_ERR_UNSUPPORTED, "beam_update: at most %d beams", kMaxBeams);
  WT_REQUIRE(hyp_slots >= 2 * beams, WT_ERR_ARG, "beam_update: hyp_slots %d < 2 * beams", hyp_slots);
  WT_REQUIRE(top_s && top_i && t && pos && sot_pos && ns && no_speech && done && hist && cum && src && tokens &&
                 forced && h_count && h_score && h_len && h_tokens && last_t,
             WT_ERR_ARG, "beam_update: null pointer");
  UpdateArgs a{top_s, top_i, t, pos, sot_pos, ns, no_speech, done, hist, cum, src, tokens, forced, h_count,
               h_score, h_len, h_tokens, last_t, sampling, samp_tok, samp_score, row_done, length, beams, capacity,
               hist_len, hyp_slots, prompt_len, vocab, eot};
  const dim3 grid(windows), block(128);
  if (beams <= 8) return launch("beam_update", beam_update_kernel<8>, grid, block, 0, stream, a);
  return launch("beam_update", beam_update_kernel<32>, grid, block, 0, stream, a);
}

int wt_beam_sample(const float *scores, const int64_t *t, const uint8_t *done, const uint8_t *row_done,
                   const uint8_t *sampling, const float *temperature, const int64_t *seed, int64_t *samp_tok,
                   float *samp_score, int windows, int beams, int vocab, void *stream) {
  using namespace wt;
  WT_REQUIRE(windows > 0 && beams > 0 && vocab > 0, WT_ERR_ARG, "beam_sample: sizes must be positive");
  WT_REQUIRE(static_cast<long long>(windows) * beams < (1LL << 31), WT_ERR_ARG, "beam_sample: too many rows");
  WT_REQUIRE(scores && t && done && row_done && sampling && temperature && seed && samp_tok && samp_score,
             WT_ERR_ARG, "beam_sample: null pointer");
  SampleArgs a{scores, t, done, row_done, sampling, temperature, seed, samp_tok, samp_score, beams, vocab};
  return launch("beam_sample", beam_sample_kernel, dim3(windows * beams), dim3(kSampleThreads), 0, stream, a);
}

int wt_slot_reset(int32_t *src, const int64_t *slots, int n_slots, int windows, int beams, int capacity,
                  int prefilled, void *stream) {
  using namespace wt;
  WT_REQUIRE(n_slots > 0 && windows > 0 && beams > 0 && capacity > 0, WT_ERR_ARG,
             "slot_reset: sizes must be positive");
  WT_REQUIRE(src && slots, WT_ERR_ARG, "slot_reset: null pointer");
  return launch("slot_reset", slot_reset_kernel, dim3(n_slots), dim3(256), 0, stream, src, slots, windows, beams,
                capacity, prefilled);
}

}  // extern "C"
