// Self-attention of S new tokens per row (a prompt), through the slot table: every new token attends to the row's
// cache slots below offset[b] -- slot j read from row src[b, j] -- and, causally, to the new tokens up to itself.
// The reference's multi-token op (whisper_trt/attn_plugin.py:102-121 body, :275-307 kernel, :462-479 launcher). It
// does not write the cache: the caller stores the new keys/values (runtime.py:177-205 copies them into new_kv).
//
// One CTA per (row, head, block of 64 queries), 4 warps of 16 queries each. Queries are the M of
// mma.sync.m16n8k16 (f32 accumulate), keys the N, the head dim the reduction; P stays in registers between
// S = Q K^T and O += P V (the S accumulator layout is the A operand layout of the next mma; P rounded to the input
// type as the reference's kernel rounds it, and for bf16 split into hi + lo parts to stay near fp32 accuracy). Key
// blocks of 64 keys are staged by cp.async into 128-byte-swizzled shared tiles (double-buffered): first the row's cache slots, each key row from the row the slot
// table names (the table's slice staged in shared memory first, so no key load waits on an index load), then the
// new tokens' keys/values straight from qkv. Out-of-range keys are zero-filled and masked; offset is clamped to
// [0, C] and slot-table rows to [0, N-1], as the reference's kernels do.
#include <type_traits>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "cross_math.cuh"

namespace wt {
namespace {

constexpr int kPD = 64;                          // head dim
constexpr int kPQ = 64;                          // queries per CTA (4 warps x 16)
constexpr int kPK = 64;                          // keys per block
constexpr int kPThreads = 128;
constexpr int kPTile = kPK * 128;                // one 64-row tile of 128-byte rows
constexpr int kPStages = 2;
constexpr int kPFixedSmem = kPTile * (1 + 2 * kPStages);  // Q tile, then (K, V) per stage; the slot-table slice after

__device__ __forceinline__ void cp_async16_zfill(void *smem_dst, const void *gmem_src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(gmem_src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kPThreads)
    self_prefill_kernel(const T *__restrict__ qkv, const T *__restrict__ kc, const T *__restrict__ vc,
                        const int64_t *__restrict__ offset, const int32_t *__restrict__ src, T *__restrict__ y,
                        int N, int S, int H, int C, float scale) {
  using E = Elem<T>;
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char *qs = smem;
  unsigned char *ring = smem + kPTile;
  int *rows_s = reinterpret_cast<int *>(smem + kPFixedSmem);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.x / H, h = blockIdx.x - (blockIdx.x / H) * H;
  const int q0 = blockIdx.y * kPQ;
  const size_t HD = static_cast<size_t>(H) * kPD, row3 = 3 * HD;
  const T *qkv_b = qkv + static_cast<size_t>(b) * S * row3;

  pdl_wait();
  pdl_launch_dependents();

  const int64_t o64 = offset[b];
  const int off = static_cast<int>(o64 < 0 ? 0 : (o64 > C ? C : o64));
  const int32_t *srow = src + static_cast<size_t>(b) * C;
  for (int i = tid; i < off; i += kPThreads) {
    const int v = srow[i];
    rows_s[i] = v < 0 ? 0 : (v > N - 1 ? N - 1 : v);
  }
  // the query tile (rows past S zero-filled)
  for (int i = tid; i < kPQ * 8; i += kPThreads) {
    const int r = i >> 3, c = i & 7, s = q0 + r;
    cp_async16_zfill(qs + swizzle128(r, c), qkv_b + static_cast<size_t>(s < S ? s : 0) * row3 + h * kPD + c * 8,
                     s < S);
  }
  __syncthreads();  // the staged slot-table slice, before the key loads that index it

  const int nbc = (off + kPK - 1) / kPK;                            // blocks of cache slots
  const int nbn = (min(S, q0 + kPQ) + kPK - 1) / kPK;               // blocks of new tokens (causal: up to this CTA)
  const int nb = nbc + nbn;

  auto load_block = [&](int kb, int stage) {
    unsigned char *kd = ring + stage * 2 * kPTile, *vd = kd + kPTile;
    for (int i = tid; i < kPK * 8; i += kPThreads) {
      const int r = i >> 3, c = i & 7;
      const T *kp, *vp;
      bool valid;
      if (kb < nbc) {
        const int j = kb * kPK + r;
        valid = j < off;
        const int jj = valid ? j : 0;
        const size_t base = ((static_cast<size_t>(valid ? rows_s[j] : b) * H + h) * C + jj) * kPD + c * 8;
        kp = kc + base;
        vp = vc + base;
      } else {
        const int j = (kb - nbc) * kPK + r;
        valid = j < S;
        kp = qkv_b + static_cast<size_t>(valid ? j : 0) * row3 + HD + h * kPD + c * 8;
        vp = kp + HD;
      }
      cp_async16_zfill(kd + swizzle128(r, c), kp, valid);
      cp_async16_zfill(vd + swizzle128(r, c), vp, valid);
    }
    cp_commit();
  };

  load_block(0, 0);  // (committed with the query tile)
  if (nb > 1) load_block(1, 1);

  const int g = lane >> 2, t = lane & 3;
  const int qw0 = q0 + warp * 16;           // this warp's first query
  const int sq0 = qw0 + g, sq1 = qw0 + g + 8;  // the two query rows this lane accumulates
  const bool active = qw0 < S;              // (a warp past the last query only helps load)
  uint32_t qa[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;

  for (int kb = 0; kb < nb; ++kb) {
    if (kb + 1 < nb) cp_wait<1>(); else cp_wait<0>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) ldmatrix_x4(qa[ks], qs + swizzle128(warp * 16 + (lane & 15), 2 * ks + (lane >> 4)));
    }
    const unsigned char *kd = ring + (kb & 1) * 2 * kPTile, *vd = kd + kPTile;
    // keys of this block: cache slots kb*64.. (valid below off) or new tokens jb.. (valid up to the query, < S)
    const bool is_new = kb >= nbc;
    const int jb = is_new ? (kb - nbc) * kPK : kb * kPK;
    // n-tiles (8 keys) that can hold a visible key for this warp: on the diagonal block, keys <= its last query
    int nact = 8;
    if (is_new) nact = min(8, max(0, (qw0 + 15 - jb) / 8 + 1));
    if (active && nact > 0) {
      float sacc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
        if (nt < nact) {
#pragma unroll
          for (int kp = 0; kp < 2; ++kp) {
            uint32_t kf[4];
            ldmatrix_x4(kf, kd + swizzle128(nt * 8 + (lane & 7), 4 * kp + (lane >> 3)));
            Mma<T>::run(sacc[nt], qa[2 * kp][0], qa[2 * kp][1], qa[2 * kp][2], qa[2 * kp][3], kf[0], kf[1]);
            Mma<T>::run(sacc[nt], qa[2 * kp + 1][0], qa[2 * kp + 1][1], qa[2 * kp + 1][2], qa[2 * kp + 1][3],
                        kf[2], kf[3]);
          }
        }
      }
      // scores in log2 units, masked: cache slots below off; new tokens up to the query and below S
      const int lim0 = is_new ? min(sq0, S - 1) : off - 1;
      const int lim1 = is_new ? min(sq1, S - 1) : off - 1;
      float mx0 = kNegInf, mx1 = kNegInf;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = jb + nt * 8 + 2 * t + e;
          sacc[nt][e] = (nt < nact && j <= lim0) ? sacc[nt][e] * scale : kNegInf;
          sacc[nt][2 + e] = (nt < nact && j <= lim1) ? sacc[nt][2 + e] * scale : kNegInf;
          mx0 = fmaxf(mx0, sacc[nt][e]);
          mx1 = fmaxf(mx1, sacc[nt][2 + e]);
        }
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float b0 = mn0 == kNegInf ? 0.f : mn0, b1 = mn1 == kNegInf ? 0.f : mn1;
      const float a0 = ex2(m0 - b0), a1 = ex2(m1 - b1);
      m0 = mn0;
      m1 = mn1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        sacc[nt][0] = ex2(sacc[nt][0] - b0);
        sacc[nt][1] = ex2(sacc[nt][1] - b0);
        sacc[nt][2] = ex2(sacc[nt][2] - b1);
        sacc[nt][3] = ex2(sacc[nt][3] - b1);
        ps0 += sacc[nt][0] + sacc[nt][1];
        ps1 += sacc[nt][2] + sacc[nt][3];
      }
      l0 = l0 * a0 + ps0;
      l1 = l1 * a1 + ps1;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        o[i][0] *= a0;
        o[i][1] *= a0;
        o[i][2] *= a1;
        o[i][3] *= a1;
      }
      // O += P V over 16 keys at a time; P in T as the reference's kernel does (attn_plugin.py:272); bf16, whose
      // 8-bit significand would cost more than the 2e-3 bar, as hi + lo
      constexpr bool kSplit = !std::is_same<T, __half>::value;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        if (2 * kk < nact) {
          uint32_t ph[4], pl[4] = {0u, 0u, 0u, 0u};
          const float *pa = sacc[2 * kk], *pb = sacc[2 * kk + 1];
          ph[0] = E::from_float2(pa[0], pa[1]);
          ph[1] = E::from_float2(pa[2], pa[3]);
          ph[2] = E::from_float2(pb[0], pb[1]);
          ph[3] = E::from_float2(pb[2], pb[3]);
          if (kSplit) {
            float2 f;
            f = E::to_float2(ph[0]);
            pl[0] = E::from_float2(pa[0] - f.x, pa[1] - f.y);
            f = E::to_float2(ph[1]);
            pl[1] = E::from_float2(pa[2] - f.x, pa[3] - f.y);
            f = E::to_float2(ph[2]);
            pl[2] = E::from_float2(pb[0] - f.x, pb[1] - f.y);
            f = E::to_float2(ph[3]);
            pl[3] = E::from_float2(pb[2] - f.x, pb[3] - f.y);
          }
#pragma unroll
          for (int dp = 0; dp < 4; ++dp) {
            uint32_t vf[4];
            ldmatrix_x4_trans(vf, vd + swizzle128(16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, 2 * dp + (lane >> 4)));
            Mma<T>::run(o[2 * dp], ph[0], ph[1], ph[2], ph[3], vf[0], vf[1]);
            Mma<T>::run(o[2 * dp + 1], ph[0], ph[1], ph[2], ph[3], vf[2], vf[3]);
            if (kSplit) {
              Mma<T>::run(o[2 * dp], pl[0], pl[1], pl[2], pl[3], vf[0], vf[1]);
              Mma<T>::run(o[2 * dp + 1], pl[0], pl[1], pl[2], pl[3], vf[2], vf[3]);
            }
          }
        }
      }
    }
    __syncthreads();  // every warp is done with this stage before it is refilled
    if (kb + 2 < nb) load_block(kb + 2, kb & 1);
  }

  if (!active) return;
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float r0 = 1.f / l0, r1 = 1.f / l1;
  // the warp's 16 output rows through its own rows of the (no longer needed) query tile, then 16-byte stores
  unsigned char *os = qs + warp * 16 * 128;
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) {
    const int byte = 4 * t;  // within the 16-byte chunk dt: head dims 8dt + 2t, +1
    *reinterpret_cast<uint32_t *>(os + swizzle128(g, dt) + byte) = E::from_float2(o[dt][0] * r0, o[dt][1] * r0);
    *reinterpret_cast<uint32_t *>(os + swizzle128(g + 8, dt) + byte) = E::from_float2(o[dt][2] * r1, o[dt][3] * r1);
  }
  __syncwarp();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = i * 32 + lane, r = idx >> 3, c = idx & 7, s = qw0 + r;
    if (s < S) {
      const uint4 v = *reinterpret_cast<const uint4 *>(os + swizzle128(r, c));
      *reinterpret_cast<uint4 *>(y + (static_cast<size_t>(b) * S + s) * HD + h * kPD + c * 8) = v;
    }
  }
}

template <typename T>
int launch_prefill(const void *qkv, const void *kc, const void *vc, const int64_t *offset, const int32_t *src,
                   void *y, int N, int S, int H, int C, void *stream) {
  auto kernel = self_prefill_kernel<T>;
  const int smem = kPFixedSmem + ((C * 4 + 127) / 128) * 128;
  const int st = opt_in_smem<self_prefill_kernel<T>>(smem, "self_attn");
  if (st != WT_OK) return st;
  const float scale = static_cast<float>(1.0 / sqrt(static_cast<double>(kPD)) * 1.4426950408889634);
  return launch("self_attn", kernel, dim3(N * H, (S + kPQ - 1) / kPQ), dim3(kPThreads), smem, stream,
                static_cast<const T *>(qkv), static_cast<const T *>(kc), static_cast<const T *>(vc), offset, src,
                static_cast<T *>(y), N, S, H, C, scale);
}

}  // namespace
}  // namespace wt

extern "C" int wt_self_attn(int dtype, const void *qkv, const void *k_cache, const void *v_cache,
                            const int64_t *offset, const int32_t *src, void *y, int rows, int new_tokens, int heads,
                            int capacity, int head_dim, void *stream) {
  using namespace wt;
  WT_REQUIRE(rows > 0 && new_tokens > 0 && heads > 0 && capacity > 0 && head_dim > 0, WT_ERR_ARG,
             "self_attn: sizes must be positive (rows %d, new_tokens %d, heads %d, capacity %d, head_dim %d)", rows,
             new_tokens, heads, capacity, head_dim);
  WT_REQUIRE(qkv && k_cache && v_cache && offset && src && y, WT_ERR_ARG, "self_attn: null pointer");
  WT_ALIGNED(qkv);
  WT_ALIGNED(k_cache);
  WT_ALIGNED(v_cache);
  WT_ALIGNED(offset);
  WT_ALIGNED(src);
  WT_ALIGNED(y);
  if (head_dim != kPD) return fail(WT_ERR_UNSUPPORTED, "self_attn: head_dim %d (supported: 64)", head_dim);
  WT_REQUIRE(static_cast<long long>(rows) * heads < (1LL << 31) && (new_tokens + kPQ - 1) / kPQ <= 65535,
             WT_ERR_ARG, "self_attn: grid too large (rows %d x heads %d, %d new tokens)", rows, heads, new_tokens);
  WT_REQUIRE(kPFixedSmem + capacity * 4LL <= 220 * 1024, WT_ERR_UNSUPPORTED,
             "self_attn: capacity %d too large for the staged slot-table slice", capacity);
  if (dtype == WT_F16)
    return launch_prefill<__half>(qkv, k_cache, v_cache, offset, src, y, rows, new_tokens, heads, capacity, stream);
  if (dtype == WT_BF16)
    return launch_prefill<__nv_bfloat16>(qkv, k_cache, v_cache, offset, src, y, rows, new_tokens, heads, capacity,
                                         stream);
  return fail(WT_ERR_DTYPE, "self_attn: unknown dtype %d", dtype);
}
