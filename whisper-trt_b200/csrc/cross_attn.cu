// Cross-attention of a window's queries (its beams / samples) over the window's encoder keys/values, split over
// the keys ("flash-decoding"), with the split partials combined by a second kernel or inside the same launch.
//
// Semantics: the reference's _cross_split_kernel / _cross_combine_kernel / _cross_attn_kernel
// (attn_plugin.py:352-435; reference bodies :129-194): scores in log2 units (scale d^-1/2 * log2 e), per key slice
// i of chunk = ceil(T / splits): m = max, p = exp2(s - m), acc = sum p v, l = sum p; combined with weights
// exp2(m_i - max m). fp16/bf16 inputs, fp32 accumulation.
//
// B200 design. HBM-bound (5 beams x 4 FLOP per key/value element pair: ~5 FLOP per byte). The one dense
// contraction of the path, so it runs on the tensor cores with warp-level mma.sync.m16n8k16 (f32 accumulate):
//   * S^T = K Q^T with the KEYS as the M dimension (16 per tile) and the window's queries as N (8 per tile, so 5
//     beams waste 3/8 instead of 11/16 with queries as M), D = 64 as the reduction (4 k-steps);
//   * O^T = V^T P^T with D as M (4 tiles) and the keys as the reduction;
//   * no shared-memory staging and no ldmatrix: the operand fragments are loaded straight from HBM with coalesced
//     16-byte loads. The key fragment uses a permutation of the head dimension (the same for the query
//     fragment, so Q.K is unchanged) that gives every lane two 16-byte pieces of its key rows; the value
//     fragment permutes D in the output (undone at the store) and pairs values of two keys with byte permutes;
//   * P goes from the S^T accumulator layout to the P^T operand layout with one movmatrix.trans per 8x8 block;
//     for bf16 inputs P is split into hi + lo bf16 parts (two mma) to keep ~16 bits of it.
// One CTA of 4 warps per (window, head, key slice, query group); each warp streams 16-key blocks of the slice
// with the next block's loads in flight while the current one is computed.
#include "cross_math.cuh"

namespace wt {

// the fused kernel (cross_stream.cu)
size_t cross_stream_workspace(int W, int S, int H, int Tn, int P);
bool cross_stream_slices_ok(int Tn, int P);
int cross_stream(int dtype, const void *q, const void *k, const void *v, void *y, int W, int S, int H, int Tn,
                 void *workspace, size_t workspace_bytes, void *stream, int P = 0, float *slices_out = nullptr);

namespace {

constexpr int kCrossWarps = 4;
constexpr int kCrossThreads = kCrossWarps * 32;

// Shared-memory layout of the CTA reduction: per warp, NT*8 queries x (64 outputs, m, l).
template <int NT>
constexpr int red_floats() {
  return kCrossWarps * NT * 8 * (kD + 2);
}

// One CTA: (window, head) = blockIdx.x, key slice = blockIdx.y, query group = blockIdx.z.
// FUSED = false: writes the reference's part[W, H, P, S, D+2] (slice partials).
// FUSED = true: writes its partial to the workspace; the last CTA of the (window, head, query group) combines all
// slices into y[W, S, H*D].
template <typename T, int NT, bool FUSED>
__global__ void __launch_bounds__(kCrossThreads)
    cross_kernel(const T *__restrict__ q, const T *__restrict__ k, const T *__restrict__ v,
                 float *__restrict__ part, int *__restrict__ counters, T *__restrict__ y, int S, int H, int Tn,
                 int P, float scale) {
  __shared__ __align__(16) float red[red_floats<NT>()];
  __shared__ int is_last;
  const int wh = blockIdx.x, sp = blockIdx.y, qg = blockIdx.z, QG = gridDim.z;
  const int w = wh / H, h = wh - w * H;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int chunk = (Tn + P - 1) / P;
  const int lo = min(Tn, sp * chunk), hi = min(Tn, lo + chunk);
  const size_t HD = static_cast<size_t>(H) * kD;
  const T *kb = k + (static_cast<size_t>(w) * H + h) * Tn * kD;
  const T *vb = v + (static_cast<size_t>(w) * H + h) * Tn * kD;
  const int q0 = qg * NT * 8;

  pdl_wait();

  uint32_t qf[NT][8];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int qi = q0 + nt * 8 + g;
    if (qi < S) {
      const T *qp = q + (static_cast<size_t>(w) * S + qi) * HD + static_cast<size_t>(h) * kD;
      const uint4 a = ldg16(qp + 8 * c), b = ldg16(qp + 32 + 8 * c);
      qf[nt][0] = a.x; qf[nt][1] = a.y; qf[nt][2] = a.z; qf[nt][3] = a.w;
      qf[nt][4] = b.x; qf[nt][5] = b.y; qf[nt][6] = b.z; qf[nt][7] = b.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) qf[nt][i] = 0u;
    }
  }
  State<NT> st;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    st.m[nt][0] = st.m[nt][1] = kNegInf;
    st.l[nt][0] = st.l[nt][1] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) st.o[nt][i][j] = 0.f;
  }

  // 16-key blocks of the slice, round-robin over the warps, two blocks in flight per warp
  constexpr int kStride = kCrossWarps * 16;
  int k0 = lo + warp * 16;
  Block cur, nxt;
  if (k0 < hi) load_block(cur, kb, vb, k0, hi, g, c);
  while (k0 < hi) {
    const int k1 = k0 + kStride;
    if (k1 < hi) load_block(nxt, kb, vb, k1, hi, g, c);
    compute_block<T, NT>(st, cur, qf, k0, hi, g, scale);
    k0 = k1;
    if (k0 >= hi) break;
    const int k2 = k0 + kStride;
    if (k2 < hi) load_block(cur, kb, vb, k2, hi, g, c);
    compute_block<T, NT>(st, nxt, qf, k0, hi, g, scale);
    k0 = k2;
  }
  pdl_launch_dependents();

  // per-warp sums over the 8 lanes of each query column, then the CTA reduction in shared memory
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) st.l[nt][j] += __shfl_xor_sync(0xffffffffu, st.l[nt][j], o);
  float *rw = red + warp * NT * 8 * (kD + 2);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float *rq = rw + (nt * 8 + 2 * c + j) * (kD + 2);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        rq[8 * g + 2 * i] = st.o[nt][i][j];      // head dim 8g+2i   (accumulator row g of tile i)
        rq[8 * g + 2 * i + 1] = st.o[nt][i][j + 2];  // head dim 8g+2i+1 (row g+8)
      }
      if (g == 0) {
        rq[kD] = st.m[nt][j];
        rq[kD + 1] = st.l[nt][j];
      }
    }
  }
  __syncthreads();

  const int nq = min(NT * 8, S - q0);  // queries of this CTA
  // combine the warps: thread -> (query, head-dim pair)
  float *outp = nullptr;
  if (FUSED) {
    outp = part + ((static_cast<size_t>(wh) * QG + qg) * P + sp) * (NT * 8) * (kD + 2);
  }
  for (int idx = tid; idx < nq * (kD / 2 + 1); idx += kCrossThreads) {
    const int qq = idx / (kD / 2 + 1), dp = idx - qq * (kD / 2 + 1);
    float top = kNegInf;
#pragma unroll
    for (int w2 = 0; w2 < kCrossWarps; ++w2) top = fmaxf(top, red[(w2 * NT * 8 + qq) * (kD + 2) + kD]);
    float n0 = 0.f, n1 = 0.f, den = 0.f;
#pragma unroll
    for (int w2 = 0; w2 < kCrossWarps; ++w2) {
      const float *rq = red + (w2 * NT * 8 + qq) * (kD + 2);
      const float mw = rq[kD];
      const float wgt = (mw == kNegInf) ? 0.f : exp2f(mw - top);
      if (dp < kD / 2) {
        n0 = fmaf(wgt, rq[2 * dp], n0);
        n1 = fmaf(wgt, rq[2 * dp + 1], n1);
      } else {
        den = fmaf(wgt, rq[kD + 1], den);
      }
    }
    float *dst = FUSED ? outp + qq * (kD + 2)
                       : part + (((static_cast<size_t>(wh) * P + sp) * S) + q0 + qq) * (kD + 2);
    if (dp < kD / 2) {
      dst[2 * dp] = n0;
      dst[2 * dp + 1] = n1;
    } else {
      dst[kD] = top;
      dst[kD + 1] = den;
    }
  }
  if (!FUSED) return;

  __threadfence();
  __syncthreads();
  const int unit = wh * QG + qg;
  if (tid == 0) is_last = (atomicAdd(counters + unit, 1) == P - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float *base = part + static_cast<size_t>(unit) * P * (NT * 8) * (kD + 2);
  for (int idx = tid; idx < nq * (kD / 8); idx += kCrossThreads) {
    const int qq = idx / (kD / 8), d8 = idx - qq * (kD / 8);
    float top = kNegInf;
    for (int s2 = 0; s2 < P; ++s2) top = fmaxf(top, __ldcg(base + (s2 * NT * 8 + qq) * (kD + 2) + kD));
    float num[8] = {0, 0, 0, 0, 0, 0, 0, 0}, den = 0.f;
    for (int s2 = 0; s2 < P; ++s2) {
      const float *ps = base + (s2 * NT * 8 + qq) * (kD + 2);
      const float ms = __ldcg(ps + kD);
      const float wgt = (ms == kNegInf) ? 0.f : exp2f(ms - top);
      den = fmaf(wgt, __ldcg(ps + kD + 1), den);
#pragma unroll
      for (int i = 0; i < 8; ++i) num[i] = fmaf(wgt, __ldcg(ps + 8 * d8 + i), num[i]);
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int i = 0; i < 8; ++i) num[i] *= inv;
    *reinterpret_cast<uint4 *>(y + (static_cast<size_t>(w) * S + q0 + qq) * HD + static_cast<size_t>(h) * kD +
                               8 * d8) = pack8<T>(num);
  }
  if (tid == 0) counters[unit] = 0;  // left zeroed for the next launch
}

// part [W, H, P, S, D+2] -> y [W, S, H*D]: one CTA per (window, head)
// The reference's combine (attn_plugin.py:182-194) of part [W, H, P, S, D + 2]: one thread per (window, head, query,
// 8-dim chunk of the output), every slice's loads of a pass of up to 8 slices issued before they are folded into a
// running (top, num, den) -- one L2 round trip per pass; slices without keys (m = -inf) weigh 0.
template <typename T>
__global__ void __launch_bounds__(128)
    combine_kernel(const float *__restrict__ part, T *__restrict__ y, int W, int S, int H, int P) {
  constexpr int kPass = 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  pdl_wait();
  // the next kernel may launch now: it reads nothing this kernel writes before its own wait, which waits for this
  // kernel to complete (so a persistent kernel after it issues its first loads while this one runs)
  pdl_launch_dependents();
  if (idx < static_cast<long long>(W) * H * S * (kD / 8)) {
    const int d8 = static_cast<int>(idx % (kD / 8));
    const long long r = idx / (kD / 8);
    const int s = static_cast<int>(r % S);
    const int wh = static_cast<int>(r / S);
    const int w = wh / H, h = wh - w * H;
    const size_t rec = kD + 2;  // (records of D + 2 floats: 8-byte aligned)
    const float *base = part + (static_cast<size_t>(wh) * P * S + s) * rec;
    float top = kNegInf, den = 0.f, num[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int i0 = 0; i0 < P; i0 += kPass) {
      float ms[kPass], ls[kPass];
      float2 a[kPass][4];
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        if (i0 + i < P) {
          const float *ps = base + static_cast<size_t>(i0 + i) * S * rec;
          const float2 ml = __ldcg(reinterpret_cast<const float2 *>(ps + kD));
          ms[i] = ml.x;
          ls[i] = ml.y;
#pragma unroll
          for (int j = 0; j < 4; ++j) a[i][j] = __ldcg(reinterpret_cast<const float2 *>(ps + 8 * d8 + 2 * j));
        } else {
          ms[i] = kNegInf;
          ls[i] = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) a[i][j] = make_float2(0.f, 0.f);
        }
      }
      float pt = top;
#pragma unroll
      for (int i = 0; i < kPass; ++i) pt = fmaxf(pt, ms[i]);
      if (pt == kNegInf) continue;  // (no keys yet)
      const float f = top == kNegInf ? 0.f : exp2f(top - pt);
      den *= f;
#pragma unroll
      for (int j = 0; j < 8; ++j) num[j] *= f;
      top = pt;
#pragma unroll
      for (int i = 0; i < kPass; ++i) {
        const float wgt = ms[i] == kNegInf ? 0.f : exp2f(ms[i] - top);
        den = fmaf(wgt, ls[i], den);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          num[2 * j] = fmaf(wgt, a[i][j].x, num[2 * j]);
          num[2 * j + 1] = fmaf(wgt, a[i][j].y, num[2 * j + 1]);
        }
      }
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int j = 0; j < 8; ++j) num[j] *= inv;
    *reinterpret_cast<uint4 *>(y + (static_cast<size_t>(w) * S + s) * static_cast<size_t>(H) * kD +
                               static_cast<size_t>(h) * kD + 8 * d8) = pack8<T>(num);
  }
}

int query_tiles(int S) {
  const int nt = (S + 7) / 8;
  return nt < 1 ? 1 : (nt > 4 ? 4 : nt);
}

// key slices of the fused kernel: about 8 CTAs per SM, at least 2 16-key blocks per warp
int fused_splits(int W, int S, int H, int Tn) {
  const int nt = query_tiles(S);
  const long long units = static_cast<long long>(W) * H * ((S + nt * 8 - 1) / (nt * 8));
  const int sms = device_sm_count();
  const long long target = static_cast<long long>(sms > 0 ? sms : 148) * 8;
  long long p = (target + units - 1) / units;
  const long long blocks = (Tn + 15) / 16;
  long long cap = blocks / (2 * kCrossWarps);
  if (cap < 1) cap = 1;
  if (p > cap) p = cap;
  if (p < 1) p = 1;
  return static_cast<int>(p);
}

float qk_scale() { return static_cast<float>(1.0 / sqrt(static_cast<double>(kD)) * 1.4426950408889634); }

template <typename T, bool FUSED>
int launch_cross(const void *q, const void *k, const void *v, float *part, int *counters, void *y, int W, int S,
                 int H, int Tn, int P, void *stream) {
  const int nt = query_tiles(S);
  const int qgs = (S + nt * 8 - 1) / (nt * 8);
  const dim3 grid(W * H, P, qgs), block(kCrossThreads);
  const T *qq = static_cast<const T *>(q), *kk = static_cast<const T *>(k), *vv = static_cast<const T *>(v);
  T *yy = static_cast<T *>(y);
  const char *what = FUSED ? "cross_attn" : "cross_attn_split";
  switch (nt) {
    case 1: return launch(what, cross_kernel<T, 1, FUSED>, grid, block, 0, stream, qq, kk, vv, part, counters, yy, S, H, Tn, P, qk_scale());
    case 2: return launch(what, cross_kernel<T, 2, FUSED>, grid, block, 0, stream, qq, kk, vv, part, counters, yy, S, H, Tn, P, qk_scale());
    case 3: return launch(what, cross_kernel<T, 3, FUSED>, grid, block, 0, stream, qq, kk, vv, part, counters, yy, S, H, Tn, P, qk_scale());
    default: return launch(what, cross_kernel<T, 4, FUSED>, grid, block, 0, stream, qq, kk, vv, part, counters, yy, S, H, Tn, P, qk_scale());
  }
}

int check_cross(const char *what, int dtype, const void *q, const void *k, const void *v, const void *out, int W,
                int S, int H, int Tn, int D) {
  WT_REQUIRE(W > 0 && S > 0 && H > 0 && Tn > 0 && D > 0, WT_ERR_ARG,
             "%s: sizes must be positive (windows %d, queries %d, heads %d, frames %d, head_dim %d)", what, W, S, H,
             Tn, D);
  WT_REQUIRE(q && k && v && out, WT_ERR_ARG, "%s: null pointer", what);
  WT_ALIGNED(q);
  WT_ALIGNED(k);
  WT_ALIGNED(v);
  WT_ALIGNED(out);
  WT_REQUIRE(D == kD, WT_ERR_UNSUPPORTED, "%s: head_dim %d (this build: 64)", what, D);
  WT_REQUIRE(dtype == WT_F16 || dtype == WT_BF16, WT_ERR_DTYPE, "%s: unknown dtype %d", what, dtype);
  WT_REQUIRE(static_cast<long long>(W) * H < (1LL << 31), WT_ERR_ARG, "%s: windows*heads too large", what);
  return WT_OK;
}

}  // namespace
}  // namespace wt

extern "C" {

int wt_cross_attn_split(int dtype, const void *q, const void *k, const void *v, float *part, int windows,
                        int queries, int heads, int frames, int head_dim, int splits, void *stream) {
  using namespace wt;
  int st = check_cross("cross_attn_split", dtype, q, k, v, part, windows, queries, heads, frames, head_dim);
  if (st != WT_OK) return st;
  WT_REQUIRE(splits > 0 && splits <= 65535, WT_ERR_ARG, "cross_attn_split: splits %d", splits);
  if (dtype == WT_F16)
    return launch_cross<__half, false>(q, k, v, part, nullptr, nullptr, windows, queries, heads, frames, splits,
                                       stream);
  return launch_cross<__nv_bfloat16, false>(q, k, v, part, nullptr, nullptr, windows, queries, heads, frames,
                                            splits, stream);
}

size_t wt_cross_attn_split_workspace(int windows, int queries, int heads, int frames, int head_dim, int splits) {
  if (windows <= 0 || queries <= 0 || heads <= 0 || frames <= 0 || head_dim != wt::kD || splits <= 0) return 0;
  if (!wt::cross_stream_slices_ok(frames, splits)) return 0;  // (the per-slice kernel, which needs none)
  return wt::cross_stream_workspace(windows, queries, heads, frames, splits);
}

int wt_cross_attn_split_ws(int dtype, const void *q, const void *k, const void *v, float *part, int windows,
                           int queries, int heads, int frames, int head_dim, int splits, void *workspace,
                           size_t workspace_bytes, void *stream) {
  using namespace wt;
  int st = check_cross("cross_attn_split", dtype, q, k, v, part, windows, queries, heads, frames, head_dim);
  if (st != WT_OK) return st;
  WT_REQUIRE(splits > 0 && splits <= 65535, WT_ERR_ARG, "cross_attn_split: splits %d", splits);
  const size_t need = wt_cross_attn_split_workspace(windows, queries, heads, frames, head_dim, splits);
  if (need == 0)
    return wt_cross_attn_split(dtype, q, k, v, part, windows, queries, heads, frames, head_dim, splits, stream);
  WT_REQUIRE(workspace && workspace_bytes >= need, WT_ERR_WORKSPACE,
             "cross_attn_split: needs a zeroed workspace of %zu bytes (given %zu)", need,
             workspace ? workspace_bytes : 0);
  WT_ALIGNED(workspace);
  return cross_stream(dtype, q, k, v, part, windows, queries, heads, frames, workspace, workspace_bytes, stream,
                      splits, part);
}

int wt_cross_attn_combine(int dtype, const float *part, void *y, int windows, int queries, int heads,
                          int head_dim, int splits, void *stream) {
  using namespace wt;
  WT_REQUIRE(windows > 0 && queries > 0 && heads > 0 && splits > 0, WT_ERR_ARG,
             "cross_attn_combine: sizes must be positive");
  WT_REQUIRE(part && y, WT_ERR_ARG, "cross_attn_combine: null pointer");
  WT_ALIGNED(part);
  WT_ALIGNED(y);
  WT_REQUIRE(head_dim == kD, WT_ERR_UNSUPPORTED, "cross_attn_combine: head_dim %d (this build: 64)", head_dim);
  const long long items = static_cast<long long>(windows) * heads * queries * (kD / 8);
  WT_REQUIRE((items + 127) / 128 < (1LL << 31), WT_ERR_ARG, "cross_attn_combine: too large");
  const dim3 grid(static_cast<unsigned>((items + 127) / 128)), block(128);
  // (after its split, not beside it: early-resident combine CTAs next to the persistent split kernel cost more
  // than the overlap gains -- measured; it still lets its successor start early)
  if (dtype == WT_F16)
    return launch_after("cross_attn_combine", combine_kernel<__half>, grid, block, 0, stream, part,
                        static_cast<__half *>(y), windows, queries, heads, splits);
  if (dtype == WT_BF16)
    return launch_after("cross_attn_combine", combine_kernel<__nv_bfloat16>, grid, block, 0, stream, part,
                        static_cast<__nv_bfloat16 *>(y), windows, queries, heads, splits);
  return fail(WT_ERR_DTYPE, "cross_attn_combine: unknown dtype %d", dtype);
}

size_t wt_cross_attn_workspace(int windows, int queries, int heads, int frames, int head_dim) {
  if (windows <= 0 || queries <= 0 || heads <= 0 || frames <= 0 || head_dim != wt::kD) return 0;
  return wt::cross_stream_workspace(windows, queries, heads, frames, 0);
}

int wt_cross_attn(int dtype, const void *q, const void *k, const void *v, void *y, int windows, int queries,
                  int heads, int frames, int head_dim, void *workspace, size_t workspace_bytes, void *stream) {
  using namespace wt;
  int st = check_cross("cross_attn", dtype, q, k, v, y, windows, queries, heads, frames, head_dim);
  if (st != WT_OK) return st;
  if (workspace) WT_ALIGNED(workspace);
  return cross_stream(dtype, q, k, v, y, windows, queries, heads, frames, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ---- wt_cross_attn_noalloc: the fused cross-attention with its scratch in a fixed device array -------------
//
// Some callers cannot allocate device memory while they run: a TensorRT-style plugin's enqueue has to work inside
// the memory its engine planned ahead of time, and an application whose device memory is owned by its own
// allocator (or that runs under a fixed memory budget) cannot let a library call cudaMalloc behind its back. For
// them this variant of wt_cross_attn takes no workspace argument: the in-kernel combine's counters and partials
// live in the array below, which every GPU that loads this library holds (8 MiB) until the process exits.

// Layout: [0, 64 KiB) one int counter per (window, head, query group); [64 KiB, 8 MiB) the slices' partials.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr size_t kNoAllocCounterBytes = size_t(64) << 10;
static __device__ __align__(256) unsigned char wt_cross_noalloc_scratch[kNoAllocScratchBytes];

#include <mutex>

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kNoAllocMaxDevices] = {};

// The device address of the scratch array on the current device, looked up once per device (the array's host-side
// name is only a stand-in: kernels need this address).
int noalloc_scratch(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return wt::fail(WT_ERR_CUDA, "cross_attn_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return wt::fail(WT_ERR_UNSUPPORTED, "cross_attn_noalloc: device %d (at most %d devices)", dev, kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, wt_cross_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return wt::fail(WT_ERR_CUDA, "cross_attn_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                      cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return WT_OK;
}

}  // namespace

extern "C" int wt_cross_attn_noalloc(int dtype, const void *q, const void *k, const void *v, void *y, int windows,
                                     int queries, int heads, int frames, int head_dim, void *stream) {
  using namespace wt;
  int st = check_cross("cross_attn_noalloc", dtype, q, k, v, y, windows, queries, heads, frames, head_dim);
  if (st != WT_OK) return st;
  const int nt = query_tiles(queries);
  const long long units = static_cast<long long>(windows) * heads * ((queries + nt * 8 - 1) / (nt * 8));
  const int P = fused_splits(windows, queries, heads, frames);
  const size_t counter_bytes = static_cast<size_t>(units) * sizeof(int);
  const size_t part_bytes = static_cast<size_t>(units) * P * nt * 8 * (kD + 2) * sizeof(float);
  WT_REQUIRE(counter_bytes <= kNoAllocCounterBytes && part_bytes <= kNoAllocScratchBytes - kNoAllocCounterBytes,
             WT_ERR_UNSUPPORTED,
             "cross_attn_noalloc: this shape needs %zu bytes of counters and %zu bytes of partials; the fixed "
             "scratch holds %zu and %zu (use wt_cross_attn with a workspace)",
             counter_bytes, part_bytes, kNoAllocCounterBytes, kNoAllocScratchBytes - kNoAllocCounterBytes);
  void *base = nullptr;
  st = noalloc_scratch(&base);
  if (st != WT_OK) return st;
  // the array keeps the previous call's contents: the counters must start at zero
  cudaError_t e = cudaMemsetAsync(base, 0, counter_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(WT_ERR_CUDA, "cross_attn_noalloc: clearing the counters: %s", cudaGetErrorString(e));
  int *counters = static_cast<int *>(base);
  float *part = reinterpret_cast<float *>(static_cast<char *>(base) + kNoAllocCounterBytes);
  if (dtype == WT_F16)
    return launch_cross<__half, true>(q, k, v, part, counters, y, windows, queries, heads, frames, P, stream);
  return launch_cross<__nv_bfloat16, true>(q, k, v, part, counters, y, windows, queries, heads, frames, P, stream);
}
