// Self-attention of one new token per row over a beam-aware KV cache read through the slot table (decode step),
// with the new token's key/value appended to the row's own cache slot.
//
// Semantics: the reference's _self_attn_step_kernel (attn_plugin.py:309-350, launcher :488-501): offset clamped
// to [0, C], slot-table entries clamped to [0, N-1], the new token attended first and always, scores in log2 units
// (scale d^-1/2 * log2 e), fp32 arithmetic on fp16/bf16 inputs, output in the input type.
//
// B200 design. The step is HBM-bound (about 1 FLOP per byte) and made of many short gathers: each (row, head)
// streams `offset` 128-byte key rows and 128-byte value rows, each from the row its slot-table entry names.
//   * one CTA of 4 warps per (row, head[, key split]); the CTA stages its slot-table slice in shared memory once
//     (so no key load waits on an index load) and its warps take 4 contiguous quarters of the keys, so the longest
//     row's chain of dependent loads is a quarter as long as with one warp per (row, head), and the many short
//     CTAs balance over the SMs by themselves;
//   * each warp streams stages of (32 / LPK) * U keys through an S-deep cp.async ring (16-byte copies, bypassing
//     L1; head_dim 64: U = 2, S = 2, 16 KB of rings per CTA): the loads in flight hold no registers, and the ring
//     is laid out piece-major ([piece][lane]) so every read-back is bank-conflict free;
//   * a key row is covered by LPK lanes (D/8 by default: one 16-byte piece each), dot products on mixed-precision
//     FMAs (half/bf16 products accumulated in fp32) finished with butterfly shuffles; each group of LPK lanes runs
//     its own online softmax (U keys per stage); groups merge by shuffles, the 4 warps through shared memory;
//   * kv_splits > 1 splits the cache capacity into equal static ranges; each split writes its partial (acc, m, l)
//     to the workspace and the last CTA of the (row, head) -- an atomic counter, no waiting -- combines them;
//   * with programmatic dependent launch the offset, slot table and cache reads start before the preceding kernel
//     has finished (only the new token's q/k/v wait for it).
#include <cstdlib>

#include "common.cuh"

namespace wt {
namespace {

constexpr int kWarpsPerCta = 4;  // key quarters of one (row, head)
constexpr int kMaxSplitKeys = 1024;  // cache slots per (row, head, split) staged in shared memory

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// acc += a * b for two packed 16-bit pairs, each product and sum in fp32 (the fp16 values convert exactly, so this
// equals unpacking then fma.f32): sm_100 mixed-precision FMA, no unpack instructions.
template <typename T> struct MixFma;
template <> struct MixFma<__half> {
  static __device__ __forceinline__ float dot2(uint32_t a, uint32_t b, float acc) {
    asm("{\n"
        ".reg .b16 alo, ahi, blo, bhi;\n"
        "mov.b32 {alo, ahi}, %1;\n"
        "mov.b32 {blo, bhi}, %2;\n"
        "fma.rn.f32.f16 %0, alo, blo, %0;\n"
        "fma.rn.f32.f16 %0, ahi, bhi, %0;\n"
        "}\n"
        : "+f"(acc)
        : "r"(a), "r"(b));
    return acc;
  }
};
template <> struct MixFma<__nv_bfloat16> {
  static __device__ __forceinline__ float dot2(uint32_t a, uint32_t b, float acc) {
    asm("{\n"
        ".reg .b16 alo, ahi, blo, bhi;\n"
        "mov.b32 {alo, ahi}, %1;\n"
        "mov.b32 {blo, bhi}, %2;\n"
        "fma.rn.f32.bf16 %0, alo, blo, %0;\n"
        "fma.rn.f32.bf16 %0, ahi, bhi, %0;\n"
        "}\n"
        : "+f"(acc)
        : "r"(a), "r"(b));
    return acc;
  }
};

__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int LPK>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = LPK / 2; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Merge two online-softmax states (m, l, acc) -> first.
template <int NA>
__device__ __forceinline__ void merge_state(float &m, float &l, float (&acc)[NA], float m2, float l2,
                                            const float (&acc2)[NA]) {
  const float mn = fmaxf(m, m2);
  const float mu = (mn == kNegInf) ? 0.f : mn;
  const float a1 = ex2(m - mu), a2 = ex2(m2 - mu);
  l = l * a1 + l2 * a2;
#pragma unroll
  for (int i = 0; i < NA; ++i) acc[i] = acc[i] * a1 + acc2[i] * a2;
  m = mn;
}

// shared memory: per warp a ring ([stage][2 * U * CPL pieces][32 lanes] x 16 bytes), then the CTA's staged source rows
template <int U, int CPL, int S>
constexpr int ring_bytes() { return S * 2 * U * CPL * 32 * 16; }

// LPK lanes cover a key row, CPL 16-byte pieces each: piece c of lane sub holds head dims (c * LPK + sub) * 8 .. + 7,
// so one copy instruction of the warp reads LPK contiguous pieces (whole 32-byte sectors) of each of its key rows.
template <typename T, int D, int LPK, int U, int kStages>
__global__ void __launch_bounds__(kWarpsPerCta * 32)
    self_step_kernel(const T *__restrict__ qkv, T *kc, T *vc, const int64_t *__restrict__ offset,
                     const int32_t *__restrict__ src, T *__restrict__ y, float *__restrict__ part,
                     int *__restrict__ counters, int N, int H, int C, int write_cache, int splits, float scale,
                     int group, int min_shared, const float *__restrict__ xrec) {
  constexpr int CPL = D / (8 * LPK);  // 16-byte pieces per lane of a key row
  constexpr int NA = 8 * CPL;         // head dims per lane
  constexpr int GPW = 32 / LPK;       // key groups per warp
  constexpr int kStageBytes = 2 * U * CPL * 32 * 16;
  constexpr int kRingBytes = ring_bytes<U, CPL, kStages>();
  constexpr int KPS = GPW * U;        // keys per stage
  static_assert(D % (8 * LPK) == 0 && 32 % LPK == 0, "lanes per key must tile the head dim and the warp");
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = blockIdx.x / H, h = blockIdx.x - (blockIdx.x / H) * H;
  const int sp = blockIdx.y;
  const int grp = lane / LPK, sub = lane % LPK;
  const size_t HD = static_cast<size_t>(H) * D;
  unsigned char *ring = smem_raw + warp * kRingBytes;
  int *rows_s = reinterpret_cast<int *>(smem_raw + kWarpsPerCta * kRingBytes);

  // Before waiting for the preceding kernel: the offset, this split's slot-table slice and the key/value rows it
  // names (inputs the kernel launched just before this one does not write; the new token's q/k/v come after).
  const int cap = (C + splits - 1) / splits;
  const int lo = sp * cap;
  const int lim = min(C, lo + cap) - lo;
  // (the whole slice, not only the slots below the offset: its loads then go out together with the offset's)
  const int64_t off64 = offset[r];
  const int32_t *srow = src + static_cast<size_t>(r) * C + lo;
  // (shared-prefix mode, xrec given, no key splits) the keys [0, p) this row shares with its group's first row a --
  // the first j below min(off, off_a) where the clamped slot tables differ, as the prefix pass finds it -- were
  // attended by that pass (the kernel launched just before this one) when p >= min_shared: this CTA takes [p, off)
  // and the new token and merges the pass's record at the end. Row a's entries are compared as the row's own are
  // staged (the same round trip).
  const int a = xrec != nullptr ? (r / group) * group : r;
  const int64_t oa64 = xrec != nullptr ? offset[a] : 0;
  const int32_t *sa = src + static_cast<size_t>(a) * C + lo;
  int mism = C;
  for (int i = threadIdx.x; i < lim; i += kWarpsPerCta * 32) {
    const int v = srow[i];
    const int cv = v < 0 ? 0 : (v > N - 1 ? N - 1 : v);
    rows_s[i] = cv;
    if (a != r) {
      const int va = sa[i];
      if ((va < 0 ? 0 : (va > N - 1 ? N - 1 : va)) != cv) mism = min(mism, i);
    }
  }
  int *p_w = rows_s + (cap + 3) / 4 * 4;  // [warp]: the warps' first mismatches
  if (xrec != nullptr) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mism = min(mism, __shfl_xor_sync(0xffffffffu, mism, o));
    if (lane == 0) p_w[warp] = mism;
  }
  const int off = static_cast<int>(off64 < 0 ? 0 : (off64 > C ? C : off64));
  __syncthreads();
  int klo = lo;
  bool shared = false;
  if (xrec != nullptr) {
    const int off_a = static_cast<int>(oa64 < 0 ? 0 : (oa64 > C ? C : oa64));
    int p = min(off, off_a);
#pragma unroll
    for (int w2 = 0; w2 < kWarpsPerCta; ++w2) p = min(p, p_w[w2]);
    shared = p >= min_shared;
    if (shared) klo = p;
  }
  const int hi = max(klo, min(off, lo + cap));  // keys [klo, hi) of this split

  // this warp's quarter: whole stages [st0, st1) of the split's range
  const int nst_all = (hi - klo + KPS - 1) / KPS;
  const int st0 = nst_all * warp / kWarpsPerCta, st1 = nst_all * (warp + 1) / kWarpsPerCta;
  const int wlo = klo + st0 * KPS, whi = min(hi, klo + st1 * KPS);
  const int nst = st1 - st0;
  const size_t row_stride = static_cast<size_t>(H) * C * D;
  const T *kh = kc + static_cast<size_t>(h) * C * D + sub * 8;
  const T *vh = vc + static_cast<size_t>(h) * C * D + sub * 8;
  // stage t: this lane's keys wlo + t*KPS + grp*U + u; piece (u, c) of K at ring[t % S][u * CPL + c][lane], of V at
  // ring[t % S][(U + u) * CPL + c][lane]
  auto issue = [&](int t) {
    unsigned char *slot = ring + (t % kStages) * kStageBytes;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = wlo + t * KPS + grp * U + u;
      if (j < whi) {
        const size_t o = static_cast<size_t>(rows_s[j - lo]) * row_stride + static_cast<size_t>(j) * D;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          cp_async16(slot + ((u * CPL + c) * 32 + lane) * 16, kh + o + c * LPK * 8);
          cp_async16(slot + (((U + u) * CPL + c) * 32 + lane) * 16, vh + o + c * LPK * 8);
        }
      }
    }
  };
#pragma unroll
  for (int t = 0; t < kStages - 1; ++t) {
    if (t < nst) issue(t);
    cp_async_commit();
  }

  pdl_wait();
  // the next kernel may launch now: it reads nothing this kernel writes before its own wait, which waits for
  // this kernel to complete
  pdl_launch_dependents();
  const T *qrow = qkv + static_cast<size_t>(r) * 3 * HD + static_cast<size_t>(h) * D + sub * 8;
  uint32_t qw[4 * CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    const uint4 qraw = ldg16(qrow + c * LPK * 8);
    qw[4 * c] = qraw.x;
    qw[4 * c + 1] = qraw.y;
    qw[4 * c + 2] = qraw.z;
    qw[4 * c + 3] = qraw.w;
  }
  // the new token first: every row attends to it (attn_plugin.py:331-334); group 0 of warp 0 of split 0 owns it
  const bool owner = sp == 0 && warp == 0;
  float m = kNegInf, l = 0.f, acc[NA];
#pragma unroll
  for (int i = 0; i < NA; ++i) acc[i] = 0.f;
  if (owner) {
    float s_new = 0.f;
    uint4 vraw[CPL];
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      const uint4 kraw = ldg16(qrow + HD + c * LPK * 8);
      vraw[c] = ldg16(qrow + 2 * HD + c * LPK * 8);
      if (write_cache && grp == 0 && off < C) {
        const size_t own = ((static_cast<size_t>(r) * H + h) * C + off) * D + sub * 8 + c * LPK * 8;
        *reinterpret_cast<uint4 *>(kc + own) = kraw;
        *reinterpret_cast<uint4 *>(vc + own) = vraw[c];
      }
      s_new = MixFma<T>::dot2(qw[4 * c], kraw.x, s_new);
      s_new = MixFma<T>::dot2(qw[4 * c + 1], kraw.y, s_new);
      s_new = MixFma<T>::dot2(qw[4 * c + 2], kraw.z, s_new);
      s_new = MixFma<T>::dot2(qw[4 * c + 3], kraw.w, s_new);
    }
    s_new = group_sum<LPK>(s_new) * scale;  // (the scale after the dot product, as attn_plugin.py:332)
    if (grp == 0) {
      m = s_new;
      l = 1.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        float vf[8];
        unpack8<T>(vraw[c], vf);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[8 * c + i] = vf[i];
      }
    }
  }

  for (int t = 0; t < nst; ++t) {
    if (t + kStages - 1 < nst) issue(t + kStages - 1);
    cp_async_commit();
    cp_async_wait<kStages - 1>();  // stage t has landed (this lane's copies)
    const unsigned char *slot = ring + (t % kStages) * kStageBytes;
    float s[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      ok[u] = wlo + t * KPS + grp * U + u < whi;
      float a = 0.f;
#pragma unroll
      for (int c = 0; c < CPL; ++c) {
        const uint4 kw = *reinterpret_cast<const uint4 *>(slot + ((u * CPL + c) * 32 + lane) * 16);
        a = MixFma<T>::dot2(qw[4 * c], kw.x, a);
        a = MixFma<T>::dot2(qw[4 * c + 1], kw.y, a);
        a = MixFma<T>::dot2(qw[4 * c + 2], kw.z, a);
        a = MixFma<T>::dot2(qw[4 * c + 3], kw.w, a);
      }
      s[u] = a;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) s[u] = group_sum<LPK>(s[u]) * scale;
    float mx = kNegInf;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      s[u] = ok[u] ? s[u] : kNegInf;
      mx = fmaxf(mx, s[u]);
    }
    const float mn = fmaxf(m, mx);
    const float mu = (mn == kNegInf) ? 0.f : mn;
    const float alpha = ex2(m - mu);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < NA; ++i) acc[i] *= alpha;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (ok[u]) {  // (a key past the range was never copied: its bytes are stale)
        const float p = ex2(s[u] - mu);
        l += p;
#pragma unroll
        for (int c = 0; c < CPL; ++c) {
          float vf[8];
          unpack8<T>(*reinterpret_cast<const uint4 *>(slot + (((U + u) * CPL + c) * 32 + lane) * 16), vf);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[8 * c + i] = fmaf(p, vf[i], acc[8 * c + i]);
        }
      }
    }
    m = mn;
  }
  cp_async_wait<0>();

  // merge the lane groups of the warp, then the warps of the CTA (through shared memory: the rings are done)
#pragma unroll
  for (int o = LPK; o < 32; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
    float acc2[NA];
#pragma unroll
    for (int i = 0; i < NA; ++i) acc2[i] = __shfl_xor_sync(0xffffffffu, acc[i], o);
    merge_state(m, l, acc, m2, l2, acc2);
  }
  __syncthreads();
  float *st_s = reinterpret_cast<float *>(smem_raw);  // [warp][D + 2]
  if (grp == 0) {
    float *mine = st_s + warp * (D + 2);
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) mine[(c * LPK + sub) * 8 + i] = acc[8 * c + i];
    if (sub == 0) {
      mine[D] = m;
      mine[D + 1] = l;
    }
  }
  __syncthreads();
  if (warp != 0 || grp != 0) return;
#pragma unroll
  for (int w2 = 1; w2 < kWarpsPerCta; ++w2) {
    const float *other = st_s + w2 * (D + 2);
    float acc2[NA];
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc2[8 * c + i] = other[(c * LPK + sub) * 8 + i];
    merge_state(m, l, acc, other[D], other[D + 1], acc2);
  }
  const int rh = r * H + h;
  T *yo = y + static_cast<size_t>(r) * HD + static_cast<size_t>(h) * D + sub * 8;
  if (shared) {  // the prefix pass's state of keys [0, p) (the kernel launched before this one, complete)
    const float *xr = xrec + static_cast<size_t>(rh) * (D + 2);
    float acc2[NA];
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int k = 0; k < 8; ++k) acc2[8 * c + k] = xr[(c * LPK + sub) * 8 + k];
    merge_state(m, l, acc, xr[D], xr[D + 1], acc2);
  }
  if (splits == 1) {
    const float inv = 1.f / l;
#pragma unroll
    for (int c = 0; c < CPL; ++c) {
      float o8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) o8[i] = acc[8 * c + i] * inv;
      *reinterpret_cast<uint4 *>(yo + c * LPK * 8) = pack8<T>(o8);
    }
    return;
  }
  // the last split of this (row, head) to finish combines the partials (lanes 0 .. LPK-1 of warp 0)
  float *pp = part + (static_cast<size_t>(rh) * splits + sp) * (D + 2);
#pragma unroll
  for (int c = 0; c < CPL; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) pp[(c * LPK + sub) * 8 + i] = acc[8 * c + i];
  if (sub == 0) {
    pp[D] = m;
    pp[D + 1] = l;
  }
  __threadfence();
  __syncwarp((1u << LPK) - 1);
  int last = 0;
  if (sub == 0) last = (atomicAdd(counters + rh, 1) == splits - 1);
  last = __shfl_sync((1u << LPK) - 1, last, 0);
  if (!last) return;
  __threadfence();
  const float *pr = part + static_cast<size_t>(rh) * splits * (D + 2);
  float top = kNegInf;
  for (int s2 = 0; s2 < splits; ++s2) top = fmaxf(top, __ldcg(pr + s2 * (D + 2) + D));
  float num[NA], den = 0.f;
#pragma unroll
  for (int i = 0; i < NA; ++i) num[i] = 0.f;
  for (int s2 = 0; s2 < splits; ++s2) {
    const float *p2 = pr + s2 * (D + 2);
    const float ms = __ldcg(p2 + D);
    const float wgt = (ms == kNegInf) ? 0.f : ex2(ms - top);
    den = fmaf(wgt, __ldcg(p2 + D + 1), den);
#pragma unroll
    for (int c = 0; c < CPL; ++c)
#pragma unroll
      for (int i = 0; i < 8; ++i) num[8 * c + i] = fmaf(wgt, __ldcg(p2 + (c * LPK + sub) * 8 + i), num[8 * c + i]);
  }
  const float inv = 1.f / den;
#pragma unroll
  for (int c = 0; c < CPL; ++c) {
    float o8[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o8[i] = num[8 * c + i] * inv;
    *reinterpret_cast<uint4 *>(yo + c * LPK * 8) = pack8<T>(o8);
  }
  if (sub == 0) counters[rh] = 0;  // left zeroed for the next launch
}

size_t step_workspace(int rows, int heads, int head_dim, int splits) {
  if (splits <= 1) return 0;
  const size_t counters = (static_cast<size_t>(rows) * heads * sizeof(int) + 255) / 256 * 256;
  return counters + static_cast<size_t>(rows) * heads * splits * (head_dim + 2) * sizeof(float);
}

template <typename T, int D, int LPK, int U, int kStages>
int launch_step(const void *qkv, void *kc, void *vc, const int64_t *offset, const int32_t *src, void *y, int N,
                int H, int C, int write_cache, int splits, void *ws, void *stream, int group, int min_shared,
                const float *xrec) {
  const int cap = (C + splits - 1) / splits;
  const int smem = kWarpsPerCta * ring_bytes<U, D / (8 * LPK), kStages>() + (cap * 4 + 15) / 16 * 16 + 16;
  auto kernel = self_step_kernel<T, D, LPK, U, kStages>;
  const int st = opt_in_smem<self_step_kernel<T, D, LPK, U, kStages>>(smem, "self_attn_step");
  if (st != WT_OK) return st;
  int *counters = nullptr;
  float *part = nullptr;
  if (splits > 1) {
    counters = static_cast<int *>(ws);
    part = reinterpret_cast<float *>(static_cast<char *>(ws) +
                                     (static_cast<size_t>(N) * H * sizeof(int) + 255) / 256 * 256);
  }
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(D)) * 1.4426950408889634);
  return launch("self_attn_step", kernel, dim3(N * H, splits), dim3(kWarpsPerCta * 32), smem, stream,
                static_cast<const T *>(qkv), static_cast<T *>(kc), static_cast<T *>(vc), offset, src,
                static_cast<T *>(y), part, counters, N, H, C, write_cache, splits, scale, group, min_shared, xrec);
}

// Shape (lanes per key row, keys per lane group per stage, stages) of the head_dim 64 kernel: (8, 2, 2) -- 16 KB of
// rings per CTA, 16 keys per warp in flight. Measured per decode step beside the 4-warp cross-attention shape
// (3 CTAs of 66.7 KB per SM): 160 rows, C 228: 1896 us against 1908 for (8, 2, 3), 1951 for (8, 4, 2), 1959 for
// (8, 1, 4), 1926 for (4, 1, 3); 80 rows, C 448, lengths U[224, 447] with the shared prefix: 1163 us against 1240
// (8, 2, 3) and 1244 (8, 4, 2); 320 rows, C 448: 4415 against 4440; 40 rows: 583 against 579. (Beside the earlier
// 8-warp cross shape, whose CTAs took 99.5 KB each, (8, 2, 3) at C <= 256 and (8, 4, 2) above had measured best.)
// Also slower at config 3: (4, 1, 2) 1938, (4, 2, 2) 1994, (8, 1, 2) 1968, (8, 1, 3) 1961 us (fewer keys in flight
// per warp, or four lanes per key row with two 16-byte pieces each). WT_SELF_SHAPE (a tuning knob) forces 0 = (8, 4, 2), 1 = (8, 2, 2),
// 2 = (8, 2, 3), 3 = (8, 1, 4) or 4 = (4, 1, 3).
int self_shape() {
  static const int forced = [] {  // (read once; a function-local static initialises thread-safely)
    const char *e = getenv("WT_SELF_SHAPE");
    const int x = e ? atoi(e) : -1;
    return (x >= 0 && x <= 4) ? x : -1;
  }();
  return forced >= 0 ? forced : 1;
}

template <typename T>
int dispatch_step(int D, const void *qkv, void *kc, void *vc, const int64_t *offset, const int32_t *src, void *y,
                  int N, int H, int C, int write_cache, int splits, void *ws, void *stream, int group = 0,
                  int min_shared = 0, const float *xrec = nullptr) {
#define WT_STEP(D_, LPK_, U_, S_)                                                                          \
  launch_step<T, D_, LPK_, U_, S_>(qkv, kc, vc, offset, src, y, N, H, C, write_cache, splits, ws, stream, group, \
                                   min_shared, xrec)
  switch (D) {
    case 16: return WT_STEP(16, 2, 4, 2);
    case 32: return WT_STEP(32, 4, 4, 2);
    case 64:
      switch (self_shape()) {
        case 1: return WT_STEP(64, 8, 2, 2);
        case 2: return WT_STEP(64, 8, 2, 3);
        case 3: return WT_STEP(64, 8, 1, 4);
        case 4: return WT_STEP(64, 4, 1, 3);
        default: return WT_STEP(64, 8, 4, 2);
      }
    case 128: return WT_STEP(128, 16, 4, 2);
    default: return fail(WT_ERR_UNSUPPORTED, "self_attn_step: head_dim %d (supported: 16, 32, 64, 128)", D);
  }
#undef WT_STEP
}

}  // namespace

int self_prefix_pass(int dtype, const void *qkv, const void *kc, const void *vc, const int64_t *offset,
                     const int32_t *src, float *rec, int N, int H, int C, int group, int min_shared, void *stream);

}  // namespace wt

extern "C" {

int wt_self_attn_step_splits(int rows, int heads, int capacity, int head_dim) {
  // one CTA of 4 warps per (row, head, split), at most 1024 slots each; split further only when the (row, head)
  // pairs alone would leave the SMs short of CTAs (< 2 per SM): splitting costs a partial and a combine
  const long long items = static_cast<long long>(rows) * heads;
  long long s = (capacity + wt::kMaxSplitKeys - 1) / wt::kMaxSplitKeys;
  const int sms = wt::device_sm_count();
  const long long want = (static_cast<long long>(sms > 0 ? sms : 148) * 2 + items - 1) / items;
  if (want > s) s = want;
  const long long cap = (capacity + 63) / 64;  // at least ~64 keys (16 per warp) per split
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return static_cast<int>(s);
}

size_t wt_self_attn_step_workspace(int rows, int heads, int head_dim, int kv_splits) {
  if (rows <= 0 || heads <= 0 || head_dim <= 0) return 0;
  return wt::step_workspace(rows, heads, head_dim, kv_splits);
}

size_t wt_self_attn_step_prefix_workspace(int rows, int heads, int head_dim) {
  if (rows <= 0 || heads <= 0 || head_dim <= 0) return 0;
  return static_cast<size_t>(rows) * heads * (head_dim + 2) * sizeof(float);
}

int wt_self_attn_step_prefix(int dtype, const void *qkv, void *k_cache, void *v_cache, const int64_t *offset,
                             const int32_t *src, void *y, int rows, int heads, int capacity, int head_dim,
                             int write_cache, int group, int min_shared, void *workspace, size_t workspace_bytes,
                             void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && heads > 0 && capacity > 0 && head_dim > 0, WT_ERR_ARG,
             "self_attn_step_prefix: sizes must be positive (rows %d, heads %d, capacity %d, head_dim %d)", rows,
             heads, capacity, head_dim);
  WT_REQUIRE(qkv && k_cache && v_cache && offset && src && y, WT_ERR_ARG, "self_attn_step_prefix: null pointer");
  WT_ALIGNED(qkv);
  WT_ALIGNED(k_cache);
  WT_ALIGNED(v_cache);
  WT_ALIGNED(offset);
  WT_ALIGNED(src);
  WT_ALIGNED(y);
  WT_REQUIRE(head_dim == 64, WT_ERR_UNSUPPORTED, "self_attn_step_prefix: head_dim %d (this build: 64)", head_dim);
  WT_REQUIRE(group >= 1 && group <= 8, WT_ERR_ARG, "self_attn_step_prefix: group %d (1-8 rows)", group);
  WT_REQUIRE(min_shared >= 1, WT_ERR_ARG, "self_attn_step_prefix: min_shared %d must be positive", min_shared);
  WT_REQUIRE(capacity <= kMaxSplitKeys, WT_ERR_UNSUPPORTED,
             "self_attn_step_prefix: capacity %d > %d (use wt_self_attn_step with key splits)", capacity,
             kMaxSplitKeys);
  WT_REQUIRE(static_cast<long long>(rows) * heads < (1LL << 31), WT_ERR_ARG,
             "self_attn_step_prefix: rows*heads too large");
  WT_REQUIRE(dtype == WT_F16 || dtype == WT_BF16, WT_ERR_DTYPE, "self_attn_step_prefix: unknown dtype %d", dtype);
  const size_t need = wt_self_attn_step_prefix_workspace(rows, heads, head_dim);
  WT_REQUIRE(workspace && workspace_bytes >= need, WT_ERR_WORKSPACE,
             "self_attn_step_prefix: needs a workspace of %zu bytes (given %zu)", need,
             workspace ? workspace_bytes : 0);
  WT_ALIGNED(workspace);
  float *rec = static_cast<float *>(workspace);
  // the prefix pass first (the shared rows' prefixes into the workspace), then the step kernel (every row's keys
  // past its shared prefix, the new token and the append, merged with the pass's record). (The other order -- the
  // step kernel's states merged by the pass -- measured slower: config 4's step 1.395 against 1.335 ms.)
  int st = self_prefix_pass(dtype, qkv, k_cache, v_cache, offset, src, rec, rows, heads, capacity, group, min_shared,
                            stream);
  if (st != WT_OK) return st;
  if (dtype == WT_F16)
    return dispatch_step<__half>(head_dim, qkv, k_cache, v_cache, offset, src, y, rows, heads, capacity, write_cache,
                                 1, nullptr, stream, group, min_shared, rec);
  return dispatch_step<__nv_bfloat16>(head_dim, qkv, k_cache, v_cache, offset, src, y, rows, heads, capacity,
                                      write_cache, 1, nullptr, stream, group, min_shared, rec);
}

int wt_self_attn_step(int dtype, const void *qkv, void *k_cache, void *v_cache, const int64_t *offset,
                      const int32_t *src, void *y, int rows, int heads, int capacity, int head_dim,
                      int write_cache, int kv_splits, void *workspace, size_t workspace_bytes, void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && heads > 0 && capacity > 0 && head_dim > 0, WT_ERR_ARG,
             "self_attn_step: sizes must be positive (rows %d, heads %d, capacity %d, head_dim %d)", rows, heads,
             capacity, head_dim);
  WT_REQUIRE(qkv && k_cache && v_cache && offset && src && y, WT_ERR_ARG, "self_attn_step: null pointer");
  WT_ALIGNED(qkv);
  WT_ALIGNED(k_cache);
  WT_ALIGNED(v_cache);
  WT_ALIGNED(offset);
  WT_ALIGNED(src);
  WT_ALIGNED(y);
  WT_REQUIRE(static_cast<long long>(rows) * heads < (1LL << 31), WT_ERR_ARG, "self_attn_step: rows*heads too large");
  int splits = kv_splits > 0 ? kv_splits : wt_self_attn_step_splits(rows, heads, capacity, head_dim);
  if (splits > capacity) splits = capacity;
  WT_REQUIRE(splits <= 65535, WT_ERR_ARG, "self_attn_step: kv_splits %d too large", splits);
  WT_REQUIRE((capacity + splits - 1) / splits <= kMaxSplitKeys, WT_ERR_ARG,
             "self_attn_step: %d cache slots per split (capacity %d / %d splits) > %d: kv_splits must be at least "
             "ceil(capacity / %d)",
             (capacity + splits - 1) / splits, capacity, splits, kMaxSplitKeys, kMaxSplitKeys);
  if (splits > 1) {
    const size_t need = step_workspace(rows, heads, head_dim, splits);
    WT_REQUIRE(workspace && workspace_bytes >= need, WT_ERR_WORKSPACE,
               "self_attn_step: %d splits need a zeroed workspace of %zu bytes (given %zu)", splits, need,
               workspace ? workspace_bytes : 0);
    WT_ALIGNED(workspace);
  }
  if (dtype == WT_F16)
    return dispatch_step<__half>(head_dim, qkv, k_cache, v_cache, offset, src, y, rows, heads, capacity,
                                 write_cache, splits, workspace, stream);
  if (dtype == WT_BF16)
    return dispatch_step<__nv_bfloat16>(head_dim, qkv, k_cache, v_cache, offset, src, y, rows, heads, capacity,
                                        write_cache, splits, workspace, stream);
  return fail(WT_ERR_DTYPE, "self_attn_step: unknown dtype %d", dtype);
}

}  // extern "C"
