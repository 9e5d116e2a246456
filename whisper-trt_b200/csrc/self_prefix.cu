// The shared-prefix pass of the decode-step self-attention: rows of a group (a window's beams or samples, `group`
// consecutive rows) whose slot tables name the same cache rows for their first positions -- the prompt every row of
// a window reads from the window's first row, the common ancestry of beams -- attend those keys together, once.
//
// Semantics: the keys [0, p_n) of row a + n of the group starting at row a, where p_n is the length of the common
// prefix of src[a + n] and src[a] (entries clamped to [0, N-1] as the step kernel reads them) below min(offset[a +
// n], offset[a]) (offsets clamped to [0, C]); a row is "shared" when p_n >= min_shared (the group's first row: p_0 =
// its offset). For every shared row the pass writes the unnormalised state of its prefix -- acc[D] (sum of
// exp2(s - m) v), m (the maximum of the log2-unit scores s = q.k * d^-1/2 * log2 e) and l (sum of exp2(s - m)) -- to
// the workspace, and the step kernel launched after it attends the row's remaining keys [p_n, offset) and the new
// token, then merges the two states (the reference's combine, attn_plugin.py:182-194): the result is the row's
// attention over all its keys, as attn_plugin.py:309-350 computes it.
//
// B200 design: one CTA of 4 warps per (group, head). The CTA finds the p_n from the group's slot tables (a block-wide
// minimum over mismatches), then its warps split the prefix's 16-key blocks in quarters: each warp gathers a
// block's key and value rows (128 bytes each, from the cache rows src[a][j] names) with 16-byte cp.async copies into
// a 128-byte-swizzled tile of its ring, zero-filled past the prefix, and runs the cross-attention's tensor-core tile
// math on it -- mma.sync with the keys as M and the group's queries as N = 8 (a window's 5 beams), P moved to the B
// operand with movmatrix -- with the key range of each query masked (keys >= p_n of query n do not count). The slot
// tables' scan and the first blocks' copies go out before the wait for the preceding kernel, the queries after it.
// The 4 warps' states merge in shared memory; 8 threads per query write the record.
#include "cross_math.cuh"
#include "tma.cuh"

namespace wt {
namespace {

constexpr int kPxWarps = 4;
constexpr int kPxStages = 4;
constexpr int kPxTile = 16 * 128;          // 16 keys x 64 elements x 2 bytes
constexpr int kPxStage = 2 * kPxTile;      // K tile + V tile
constexpr int kPxRec = kD + 2;             // acc[64], m, l
constexpr int kPxMaxGroup = 8;             // queries of a group (the MMA's N)

__device__ __forceinline__ void cp_async16_zfill(void *smem_dst, const void *gmem_src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem_dst)), "l"(gmem_src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void px_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void px_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// One 16-key block into the online-softmax state of the group's 8 query columns, each element masked by its own
// condition: v0 (key g, query 2c), v1 (key g, query 2c + 1), v2 (key g + 8, query 2c), v3 (key g + 8, query 2c + 1).
// A column with no key yet keeps m = -inf (the rescale of an empty state is skipped, as merge_state does).
template <typename T>
__device__ __forceinline__ void attend_block_cols(State<1> &st, const uint32_t (&ka)[4][4],
                                                  const uint32_t (&va)[4][4], const uint32_t (&qf)[1][8], bool v0,
                                                  bool v1, bool v2, bool v3, float scale) {
  float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int s = 0; s < 4; ++s) Mma<T>::run(sc, ka[s][0], ka[s][1], ka[s][2], ka[s][3], qf[0][2 * s], qf[0][2 * s + 1]);
  const float s0 = v0 ? sc[0] * scale : kNegInf, s1 = v1 ? sc[1] * scale : kNegInf;
  const float s2 = v2 ? sc[2] * scale : kNegInf, s3 = v3 ? sc[3] * scale : kNegInf;
  float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
  }
  const float mn0 = fmaxf(st.m[0][0], mx0), mn1 = fmaxf(st.m[0][1], mx1);
  const float mu0 = mn0 == kNegInf ? 0.f : mn0, mu1 = mn1 == kNegInf ? 0.f : mn1;
  const float a0 = ex2(st.m[0][0] - mu0), a1 = ex2(st.m[0][1] - mu1);  // (ex2(-inf) = 0: an empty state)
  st.m[0][0] = mn0;
  st.m[0][1] = mn1;
  const float p0 = ex2(s0 - mu0), p1 = ex2(s1 - mu1), p2 = ex2(s2 - mu0), p3 = ex2(s3 - mu1);
  // P as hi + lo parts in the input type (two products), the row sums from the same split values
  const uint32_t h01 = Elem<T>::from_float2(p0, p1), h23 = Elem<T>::from_float2(p2, p3);
  const float2 r01 = Elem<T>::to_float2(h01), r23 = Elem<T>::to_float2(h23);
  const uint32_t lo01 = Elem<T>::from_float2(p0 - r01.x, p1 - r01.y), lo23 = Elem<T>::from_float2(p2 - r23.x, p3 - r23.y);
  const float2 q01 = Elem<T>::to_float2(lo01), q23 = Elem<T>::to_float2(lo23);
  st.l[0][0] = st.l[0][0] * a0 + (r01.x + r23.x + q01.x + q23.x);
  st.l[0][1] = st.l[0][1] * a1 + (r01.y + r23.y + q01.y + q23.y);
  const uint32_t pb0 = movmatrix_trans(h01), pb1 = movmatrix_trans(h23);
  const uint32_t qb0 = movmatrix_trans(lo01), qb1 = movmatrix_trans(lo23);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    st.o[0][i][0] *= a0;
    st.o[0][i][1] *= a1;
    st.o[0][i][2] *= a0;
    st.o[0][i][3] *= a1;
    Mma<T>::run(st.o[0][i], va[i][0], va[i][1], va[i][2], va[i][3], pb0, pb1);
    Mma<T>::run(st.o[0][i], va[i][0], va[i][1], va[i][2], va[i][3], qb0, qb1);
  }
}

// shared memory: per warp a ring of kPxStages (K, V) tiles, then the warps' states [warp][8 queries][kPxRec], then the
// anchor row's clamped slot table [C], then the group's prefix lengths [8]
template <typename T>
__global__ void __launch_bounds__(kPxWarps * 32)
    self_prefix_kernel(const T *__restrict__ qkv, const T *__restrict__ kc, const T *__restrict__ vc,
                       const int64_t *__restrict__ offset, const int32_t *__restrict__ src, float *__restrict__ rec,
                       int N, int H, int C, int group, int min_shared, float scale) {
  extern __shared__ unsigned char px_raw[];
  unsigned char *px_smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(px_raw) + 127) & ~uintptr_t(127));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int gi = blockIdx.x / H, h = blockIdx.x - (blockIdx.x / H) * H;
  const int a = gi * group, ng = min(group, N - a);
  unsigned char *ring = px_smem + warp * kPxStages * kPxStage;
  float *st_s = reinterpret_cast<float *>(px_smem + kPxWarps * kPxStages * kPxStage);
  int *src_a = reinterpret_cast<int *>(st_s + kPxWarps * kPxMaxGroup * kPxRec);
  int *plen = src_a + C;

  // the group's prefix lengths: p_n = the first j below min(off[a + n], off[a]) where the clamped slot-table
  // entries of rows a + n and a differ (inputs the kernel launched just before this one does not write)
  auto clamp_row = [N](int v) { return v < 0 ? 0 : (v > N - 1 ? N - 1 : v); };
  auto clamp_off = [C](int64_t v) { return static_cast<int>(v < 0 ? 0 : (v > C ? C : v)); };
  const int off_a = clamp_off(offset[a]);
  // every member's shared prefix lies in the first row's keys [0, off_a), which the first row itself shares whole:
  // nothing to do below min_shared (uniform over the CTA), else those keys are the ones to gather
  if (off_a < min_shared) return;
  if (threadIdx.x < kPxMaxGroup) plen[threadIdx.x] = threadIdx.x < ng ? min(clamp_off(offset[a + threadIdx.x]), off_a) : 0;
  const int32_t *sa = src + static_cast<size_t>(a) * C;
  // the members' entries in 4-entry chunks, (member, chunk) pairs spread over the threads, four loads in flight per
  // thread, the first four issued with the first row's: one round trip for a group of up to 4 members at C <= 448
  // (the rows are 16-byte aligned when C is a multiple of 4; otherwise one entry at a time)
  const bool vec = C % 4 == 0;
  const int nq = C / 4, total = vec ? (ng - 1) * nq : 0;
  constexpr int kStride = kPxWarps * 32;
  int4 v[4];
  auto load4 = [&](int i0) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int i = i0 + u * kStride;
      if (i < total) {
        const int n = 1 + i / nq, q = i - (i / nq) * nq;
        v[u] = __ldg(reinterpret_cast<const int4 *>(src + static_cast<size_t>(a + n) * C) + q);
      }
    }
  };
  load4(threadIdx.x);
  for (int j = threadIdx.x; j < C; j += kStride) src_a[j] = clamp_row(sa[j]);
  __syncthreads();
  // this warp's 16-key blocks [b0, b1) of the prefix; the first stages' copies go out now, the members' scan (which
  // sets each query's key range, not the keys) runs while they are in flight
  const int pmax = off_a;
  const int nblk = (pmax + 15) / 16;
  const int b0 = nblk * warp / kPxWarps, b1 = nblk * (warp + 1) / kPxWarps;
  const int nw = b1 - b0;
  const size_t row_stride = static_cast<size_t>(H) * C * kD;
  const T *kh = kc + static_cast<size_t>(h) * C * kD;
  const T *vh = vc + static_cast<size_t>(h) * C * kD;
  // block b into stage s: lane covers rows lane / 8 + 4 i (i < 4), 16-byte chunk lane % 8 of each, swizzled
  auto issue = [&](int b, int s) {
    unsigned char *kt = ring + s * kPxStage, *vt = kt + kPxTile;
    const int ch = lane & 7;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rr = (lane >> 3) + 4 * i, j = b * 16 + rr;
      const bool ok = j < pmax;
      const size_t o = ok ? static_cast<size_t>(src_a[j]) * row_stride + static_cast<size_t>(j) * kD + ch * 8 : 0;
      cp_async16_zfill(kt + swizzle128(rr, ch), kh + o, ok);
      cp_async16_zfill(vt + swizzle128(rr, ch), vh + o, ok);
    }
  };
#pragma unroll
  for (int s = 0; s < kPxStages - 1; ++s) {
    if (s < nw) issue(b0 + s, s);
    px_commit();
  }

  if (vec) {
    for (int i0 = threadIdx.x; i0 < total; i0 += 4 * kStride) {
      if (i0 != static_cast<int>(threadIdx.x)) load4(i0);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * kStride;
        if (i < total) {
          const int n = 1 + i / nq, jj = 4 * (i - (i / nq) * nq);
          const int lim = plen[n];
          const int e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
          int first = C;
#pragma unroll
          for (int k = 3; k >= 0; --k)
            if (jj + k < lim && clamp_row(e[k]) != src_a[jj + k]) first = jj + k;
          if (first < C) atomicMin(&plen[n], first);
        }
      }
    }
  } else {
    for (int n = 1; n < ng; ++n) {
      const int32_t *sn = src + static_cast<size_t>(a + n) * C;
      const int lim = plen[n];
      for (int jj = threadIdx.x; jj < lim; jj += kStride)
        if (clamp_row(sn[jj]) != src_a[jj]) atomicMin(&plen[n], jj);
    }
  }
  __syncthreads();
  // a query column takes part when its row is shared: keys [0, lim) of column n
  const int nb = (2 * c < ng && plen[2 * c] >= min_shared) ? plen[2 * c] : 0;
  const int nb1 = (2 * c + 1 < ng && plen[2 * c + 1] >= min_shared) ? plen[2 * c + 1] : 0;

  pdl_wait();
  pdl_launch_dependents();
  const size_t HD3 = static_cast<size_t>(3) * H * kD;
  uint32_t qf[1][8];
  load_q_std<T, 1>(qf, qkv + static_cast<size_t>(a) * HD3 + static_cast<size_t>(h) * kD, HD3, 0, ng, g, c);
  State<1> st;
  st.m[0][0] = st.m[0][1] = kNegInf;
  st.l[0][0] = st.l[0][1] = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) st.o[0][i][k] = 0.f;
  for (int t = 0; t < nw; ++t) {
    if (t + kPxStages - 1 < nw) issue(b0 + t + kPxStages - 1, (t + kPxStages - 1) % kPxStages);
    px_commit();
    px_wait<kPxStages - 1>();  // block t has landed (this lane's copies) ...
    __syncwarp();              // ... and every lane's
    const unsigned char *kt = ring + (t % kPxStages) * kPxStage;
    uint32_t ka[4][4], va[4][4];
    smem_frags(ka, va, kt, kt + kPxTile, lane);
    __syncwarp();  // (every lane's reads of this stage before any lane's copies refill it: one proxy, the generic)
    const int k0 = (b0 + t) * 16;
    attend_block_cols<T>(st, ka, va, qf, k0 + g < nb, k0 + g < nb1, k0 + g + 8 < nb, k0 + g + 8 < nb1, scale);
  }
  px_wait<0>();

  // this warp's state -> shared memory, one record per query column (the row sums reduced over the lanes)
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) st.l[0][j] += __shfl_xor_sync(0xffffffffu, st.l[0][j], o);
  float *mine = st_s + warp * kPxMaxGroup * kPxRec;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float *rq = mine + (2 * c + j) * kPxRec;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rq[16 * i + g] = st.o[0][i][j];
      rq[16 * i + g + 8] = st.o[0][i][j + 2];
    }
    if (g == 0) {
      rq[kD] = st.m[0][j];
      rq[kD + 1] = st.l[0][j];
    }
  }
  __syncthreads();
  // the warps' states -> each shared row's record: thread t takes query t / 8, head dims 8 (t % 8) .. + 7
  if (threadIdx.x < kPxMaxGroup * 8) {
    const int n = threadIdx.x >> 3, d8 = threadIdx.x & 7;
    if (n < ng && plen[n] >= min_shared) {
      float top = kNegInf;
#pragma unroll
      for (int w2 = 0; w2 < kPxWarps; ++w2) top = fmaxf(top, st_s[(w2 * kPxMaxGroup + n) * kPxRec + kD]);
      const float mu = top == kNegInf ? 0.f : top;
      float den = 0.f, num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w2 = 0; w2 < kPxWarps; ++w2) {
        const float *r = st_s + (w2 * kPxMaxGroup + n) * kPxRec;
        const float wgt = r[kD] == kNegInf ? 0.f : ex2(r[kD] - mu);
        den = fmaf(wgt, r[kD + 1], den);
#pragma unroll
        for (int i = 0; i < 8; ++i) num[i] = fmaf(wgt, r[8 * d8 + i], num[i]);
      }
      float *out = rec + (static_cast<size_t>(a + n) * H + h) * kPxRec;
#pragma unroll
      for (int i = 0; i < 8; ++i) out[8 * d8 + i] = num[i];
      if (d8 == 0) {
        out[kD] = top;
        out[kD + 1] = den;
      }
    }
  }
}

template <typename T>
int launch_prefix(const void *qkv, const void *kc, const void *vc, const int64_t *offset, const int32_t *src,
                  float *rec, int N, int H, int C, int group, int min_shared, void *stream) {
  const int smem =
      128 + kPxWarps * kPxStages * kPxStage + kPxWarps * kPxMaxGroup * kPxRec * 4 + C * 4 + kPxMaxGroup * 4;
  const int st = opt_in_smem<self_prefix_kernel<T>>(smem, "self_attn_step (shared prefix)");
  if (st != WT_OK) return st;
  const int groups = (N + group - 1) / group;
  const float scale = static_cast<float>(1.0 / 8.0 * 1.4426950408889634);
  return launch("self_attn_step (shared prefix)", self_prefix_kernel<T>, dim3(groups * H), dim3(kPxWarps * 32), smem,
                stream, static_cast<const T *>(qkv), static_cast<const T *>(kc), static_cast<const T *>(vc), offset,
                src, rec, N, H, C, group, min_shared, scale);
}

}  // namespace

// The shared-prefix pass for head_dim 64 (the records of every shared row, [N, H, D + 2] floats at `rec`).
int self_prefix_pass(int dtype, const void *qkv, const void *kc, const void *vc, const int64_t *offset,
                     const int32_t *src, float *rec, int N, int H, int C, int group, int min_shared, void *stream) {
  if (dtype == WT_BF16)
    return launch_prefix<__nv_bfloat16>(qkv, kc, vc, offset, src, rec, N, H, C, group, min_shared, stream);
  return launch_prefix<__half>(qkv, kc, vc, offset, src, rec, N, H, C, group, min_shared, stream);
}

}  // namespace wt
