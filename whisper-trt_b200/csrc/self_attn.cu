// Self-attention of one new token per row over a beam-aware KV cache read through the slot table (decode step),
// with the new token's key/value appended to the row's own cache slot.
//
// Semantics: the reference's _self_attn_step_kernel (attn_plugin.py:309-350, launcher :488-501): offset clamped
// to [0, C], slot-table entries clamped to [0, N-1], the new token attended first and always, scores in log2 units
// (scale d^-1/2 * log2 e), fp32 arithmetic on fp16/bf16 inputs, output in the input type.
//
// B200 design. The step is HBM-bound (about 1 FLOP per byte): each (row, head) streams `offset` gathered 128-byte
// key rows and 128-byte value rows. One CTA of 4 warps per (row, head[, key split]):
//   * the CTA's slot-table entries are staged in shared memory once, so every key/value load is issued without
//     waiting on a dependent index load;
//   * a key row is read by D/8 lanes with one 16-byte vector load each (a warp reads 4 whole 128-byte rows per
//     instruction: every byte of every fetched sector is used); each lane keeps the matching 8 query elements, the
//     dot product is finished with 3 butterfly shuffles;
//   * each group of D/8 lanes runs its own online softmax over 4 keys per iteration, the groups and warps are
//     merged at the end (shuffles, then shared memory);
//   * kv_splits > 1 splits a row's cache range over CTAs; each writes its partial (acc, m, l) to the workspace and
//     the last CTA of the (row, head) -- found with an atomic counter, no waiting -- combines them.
#include "common.cuh"

namespace wt {
namespace {

constexpr int kSelfWarps = 4;
constexpr int kSelfThreads = kSelfWarps * 32;
constexpr int kKeysPerGroup = 4;  // keys per lane group per iteration
constexpr int kMaxCapacity = 16384;

template <int LPK>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int o = LPK / 2; o >= 1; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Merge two online-softmax states (m, l, acc) -> first.
__device__ __forceinline__ void merge_state(float &m, float &l, float (&acc)[8], float m2, float l2,
                                            const float (&acc2)[8]) {
  const float mn = fmaxf(m, m2);
  const float mu = (mn == kNegInf) ? 0.f : mn;
  const float a1 = exp2f(m - mu), a2 = exp2f(m2 - mu);
  l = l * a1 + l2 * a2;
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = acc[i] * a1 + acc2[i] * a2;
  m = mn;
}

template <typename T, int D>
__global__ void __launch_bounds__(kSelfThreads)
    self_step_kernel(const T *__restrict__ qkv, T *kc, T *vc, const int64_t *__restrict__ offset,
                     const int32_t *__restrict__ src, T *__restrict__ y, float *__restrict__ part,
                     int *__restrict__ counters, int N, int H, int C, int write_cache, int splits, float scale) {
  constexpr int LPK = D / 8;          // lanes per key row (16 bytes each)
  constexpr int GPW = 32 / LPK;       // key groups per warp
  constexpr int U = kKeysPerGroup;
  constexpr int KPW = GPW * U;        // keys per warp per iteration
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float *red = reinterpret_cast<float *>(smem_raw);                      // [warps][D + 2]
  int *rows_s = reinterpret_cast<int *>(red + kSelfWarps * (D + 2));      // [range] source rows

  const int rh = blockIdx.x, sp = blockIdx.y;
  const int r = rh / H, h = rh - r * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int grp = lane / LPK, sub = lane % LPK;
  const size_t HD = static_cast<size_t>(H) * D;

  pdl_wait();

  const int64_t off64 = offset[r];
  const int off = static_cast<int>(off64 < 0 ? 0 : (off64 > C ? C : off64));
  const int per = (off + splits - 1) / splits;
  const int lo = min(off, sp * per), hi = min(off, lo + per);

  const int32_t *srow = src + static_cast<size_t>(r) * C;
  for (int i = tid; i < hi - lo; i += kSelfThreads) {
    const int v = srow[lo + i];
    rows_s[i] = v < 0 ? 0 : (v > N - 1 ? N - 1 : v);
  }

  const T *qrow = qkv + static_cast<size_t>(r) * 3 * HD + static_cast<size_t>(h) * D + sub * 8;
  const uint4 qraw = ldg16(qrow), kraw = ldg16(qrow + HD), vraw = ldg16(qrow + 2 * HD);
  if (write_cache && sp == 0 && warp == 0 && grp == 0 && off < C) {
    const size_t own = ((static_cast<size_t>(r) * H + h) * C + off) * D + sub * 8;
    *reinterpret_cast<uint4 *>(kc + own) = kraw;
    *reinterpret_cast<uint4 *>(vc + own) = vraw;
  }
  float q[8], kn[8];
  unpack8<T>(qraw, q);
  unpack8<T>(kraw, kn);
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] *= scale;
  float s_new = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s_new = fmaf(q[i], kn[i], s_new);
  s_new = group_sum<LPK>(s_new);

  // the new token first: every row attends to it (attn_plugin.py:331-334); one group of one CTA owns it
  float m = kNegInf, l = 0.f, acc[8];
  if (sp == 0 && warp == 0 && grp == 0) {
    m = s_new;
    l = 1.f;
    unpack8<T>(vraw, acc);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  }
  __syncthreads();

  const size_t row_stride = static_cast<size_t>(H) * C * D;
  const T *kh = kc + static_cast<size_t>(h) * C * D + sub * 8;
  const T *vh = vc + static_cast<size_t>(h) * C * D + sub * 8;
  for (int k0 = lo + warp * KPW; k0 < hi; k0 += kSelfWarps * KPW) {
    uint4 kr[U], vr[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = k0 + grp * U + u;
      ok[u] = j < hi;
      if (ok[u]) {
        const size_t o = static_cast<size_t>(rows_s[j - lo]) * row_stride + static_cast<size_t>(j) * D;
        kr[u] = ldg_stream(kh + o);
        vr[u] = ldg_stream(vh + o);
      } else {
        kr[u] = make_uint4(0, 0, 0, 0);
        vr[u] = kr[u];
      }
    }
    float s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float kf[8];
      unpack8<T>(kr[u], kf);
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) a = fmaf(q[i], kf[i], a);
      s[u] = a;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) s[u] = group_sum<LPK>(s[u]);
    float mx = kNegInf;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      s[u] = ok[u] ? s[u] : kNegInf;
      mx = fmaxf(mx, s[u]);
    }
    const float mn = fmaxf(m, mx);
    const float mu = (mn == kNegInf) ? 0.f : mn;
    const float alpha = exp2f(m - mu);
    l *= alpha;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] *= alpha;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float p = exp2f(s[u] - mu);
      l += p;
      float vf[8];
      unpack8<T>(vr[u], vf);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(p, vf[i], acc[i]);
    }
    m = mn;
  }
  pdl_launch_dependents();

  // merge the lane groups of the warp
#pragma unroll
  for (int o = LPK; o < 32; o <<= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o), l2 = __shfl_xor_sync(0xffffffffu, l, o);
    float acc2[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc2[i] = __shfl_xor_sync(0xffffffffu, acc[i], o);
    merge_state(m, l, acc, m2, l2, acc2);
  }
  // merge the warps
  if (grp == 0) {
    float *rw = red + warp * (D + 2);
#pragma unroll
    for (int i = 0; i < 8; ++i) rw[sub * 8 + i] = acc[i];
    if (sub == 0) {
      rw[D] = m;
      rw[D + 1] = l;
    }
  }
  __syncthreads();
  if (warp == 0 && grp == 0) {
    for (int w2 = 1; w2 < kSelfWarps; ++w2) {
      const float *rw = red + w2 * (D + 2);
      float acc2[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc2[i] = rw[sub * 8 + i];
      merge_state(m, l, acc, rw[D], rw[D + 1], acc2);
    }
    if (splits == 1) {
      const float inv = 1.f / l;
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] *= inv;
      *reinterpret_cast<uint4 *>(y + static_cast<size_t>(r) * HD + static_cast<size_t>(h) * D + sub * 8) =
          pack8<T>(acc);
    } else {
      float *pp = part + (static_cast<size_t>(rh) * splits + sp) * (D + 2);
#pragma unroll
      for (int i = 0; i < 8; ++i) pp[sub * 8 + i] = acc[i];
      if (sub == 0) {
        pp[D] = m;
        pp[D + 1] = l;
      }
    }
  }
  if (splits == 1) return;

  // the last CTA of this (row, head) combines the splits' partials
  __shared__ int is_last;
  __threadfence();
  __syncthreads();
  if (tid == 0) is_last = (atomicAdd(counters + rh, 1) == splits - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  if (warp == 0 && grp == 0) {
    const float *pr = part + static_cast<size_t>(rh) * splits * (D + 2);
    float top = kNegInf;
    for (int s2 = 0; s2 < splits; ++s2) top = fmaxf(top, __ldcg(pr + s2 * (D + 2) + D));
    float num[8] = {0, 0, 0, 0, 0, 0, 0, 0}, den = 0.f;
    for (int s2 = 0; s2 < splits; ++s2) {
      const float *p2 = pr + s2 * (D + 2);
      const float ms = __ldcg(p2 + D);
      const float wgt = (ms == kNegInf) ? 0.f : exp2f(ms - top);
      den = fmaf(wgt, __ldcg(p2 + D + 1), den);
#pragma unroll
      for (int i = 0; i < 8; ++i) num[i] = fmaf(wgt, __ldcg(p2 + sub * 8 + i), num[i]);
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int i = 0; i < 8; ++i) num[i] *= inv;
    *reinterpret_cast<uint4 *>(y + static_cast<size_t>(r) * HD + static_cast<size_t>(h) * D + sub * 8) =
        pack8<T>(num);
  }
  if (tid == 0) counters[rh] = 0;  // left zeroed for the next launch
}

size_t step_workspace(int rows, int heads, int head_dim, int splits) {
  if (splits <= 1) return 0;
  const size_t counters = (static_cast<size_t>(rows) * heads * sizeof(int) + 255) / 256 * 256;
  return counters + static_cast<size_t>(rows) * heads * splits * (head_dim + 2) * sizeof(float);
}

template <typename T, int D>
int launch_step(const void *qkv, void *kc, void *vc, const int64_t *offset, const int32_t *src, void *y, int N,
                int H, int C, int write_cache, int splits, void *ws, void *stream) {
  const int range = (C + splits - 1) / splits;
  const size_t smem = kSelfWarps * (D + 2) * sizeof(float) + static_cast<size_t>(range) * sizeof(int);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(self_step_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kSelfWarps * (D + 2) * 4 + kMaxCapacity * 4);
    attr_set = true;
  }
  int *counters = nullptr;
  float *part = nullptr;
  if (splits > 1) {
    counters = static_cast<int *>(ws);
    part = reinterpret_cast<float *>(static_cast<char *>(ws) +
                                     (static_cast<size_t>(N) * H * sizeof(int) + 255) / 256 * 256);
  }
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(D)) * 1.4426950408889634);
  return launch("self_attn_step", self_step_kernel<T, D>, dim3(N * H, splits), dim3(kSelfThreads), smem, stream,
                static_cast<const T *>(qkv), static_cast<T *>(kc), static_cast<T *>(vc), offset, src,
                static_cast<T *>(y), part, counters, N, H, C, write_cache, splits, scale);
}

template <typename T>
int dispatch_step(int D, const void *qkv, void *kc, void *vc, const int64_t *offset, const int32_t *src, void *y,
                  int N, int H, int C, int write_cache, int splits, void *ws, void *stream) {
  switch (D) {
    case 16: return launch_step<T, 16>(qkv, kc, vc, offset, src, y, N, H, C, write_cache, splits, ws, stream);
    case 32: return launch_step<T, 32>(qkv, kc, vc, offset, src, y, N, H, C, write_cache, splits, ws, stream);
    case 64: return launch_step<T, 64>(qkv, kc, vc, offset, src, y, N, H, C, write_cache, splits, ws, stream);
    case 128: return launch_step<T, 128>(qkv, kc, vc, offset, src, y, N, H, C, write_cache, splits, ws, stream);
    default: return fail(WT_ERR_UNSUPPORTED, "self_attn_step: head_dim %d (supported: 16, 32, 64, 128)", D);
  }
}

}  // namespace
}  // namespace wt

extern "C" {

int wt_self_attn_step_splits(int rows, int heads, int capacity, int head_dim) {
  // one CTA per (row, head) already gives >= 4 CTAs of 4 warps per SM on 148 SMs: no split
  const long long ctas = static_cast<long long>(rows) * heads;
  const long long target = 148LL * 4;
  if (ctas >= target || capacity <= 64) return 1;
  long long s = (target + ctas - 1) / ctas;
  const long long cap = capacity / 32;  // at least ~32 keys per split
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  if (s > 64) s = 64;
  return static_cast<int>(s);
}

size_t wt_self_attn_step_workspace(int rows, int heads, int head_dim, int kv_splits) {
  if (rows <= 0 || heads <= 0 || head_dim <= 0) return 0;
  return wt::step_workspace(rows, heads, head_dim, kv_splits);
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
  WT_REQUIRE(capacity <= kMaxCapacity, WT_ERR_UNSUPPORTED, "self_attn_step: capacity %d > %d", capacity,
             kMaxCapacity);
  WT_REQUIRE(static_cast<long long>(rows) * heads < (1LL << 31), WT_ERR_ARG, "self_attn_step: rows*heads too large");
  int splits = kv_splits > 0 ? kv_splits : wt_self_attn_step_splits(rows, heads, capacity, head_dim);
  if (splits > capacity) splits = capacity;
  WT_REQUIRE(splits <= 65535, WT_ERR_ARG, "self_attn_step: kv_splits %d too large", splits);
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
