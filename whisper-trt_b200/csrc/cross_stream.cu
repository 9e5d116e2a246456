// Fused cross-attention (split + combine in one launch), fed by TMA: a window of at most 8 queries (a beam or a
// sample group) takes cross_window_kernel below -- one CTA per (window, head), 4 or 8 key slices combined in shared
// memory; larger query groups, and the reference-shaped split (slice mode), take the persistent stream-K kernel.
//
// Semantics: the reference's cross_attn (attn_plugin.py:129-136, kernel :352-376) -- softmax(q k^T / sqrt(D)) v per
// (window, head) over the window's T encoder frames, scores in log2 units; fp32 accumulation.
//
// The stream-K kernel. The work is the flat sequence of (window, head, query group, 16-key block) units -- 94 blocks per
// (window, head) at T = 1500 -- cut into one equal contiguous range per streaming warp of a persistent grid
// ("stream-K": every warp streams the same number of bytes, no wave tail whatever the window count):
//   * each streaming warp owns a ring of stages in shared memory; its lane 0 issues 2D TMA loads (16 rows x 128 bytes
//     of K and of V, 128-byte swizzle) that complete on the stage's mbarrier, keeping the other stages in flight
//     while the warp computes -- no registers are held by loads in flight;
//   * the block's mma operands are read from the swizzled tile with bank-conflict-free 16-byte shared loads and
//     go through the same tensor-core math as the split kernel (cross_math.cuh);
//   * a unit wholly inside one warp's range goes straight to the output; the range's first and last units are shared
//     with the neighbouring warps: the warp stores its partial (acc, m, l) for them, their counters count the blocks
//     done, and the warp that completes a unit -- no waiting -- combines its partials (at most
//     ceil(94 / blocks per warp) + 1) into the output;
//   * a streaming warp never executes a GPU-scope fence while its loads are in flight: such a fence (which a count
//     needs after the partial's stores) stalled the warp for about as long as eight blocks take to stream. The first
//     unit's count, due in mid-range, is left to the CTA's one service warp, which issues no loads: the streaming
//     warp stores its partial and arrives on an mbarrier (a CTA-scope release), and the service warp fences and
//     counts. The last unit is counted by its warp at the end of its range, when nothing of its own is in flight.
// Every mbarrier wait is bounded: a wait that times out records an error code in the workspace, and the warp stops
// streaming, waits (bounded) for the copies it still has in flight and leaves its units unfinished.
// With programmatic dependent launch the first TMA loads are issued before the preceding kernel has finished (the
// cross keys/values are not its output); the queries are read after it, one unit ahead of their use.
#include <cstdlib>

#include "cross_math.cuh"
#include "tma.cuh"

namespace wt {

bool cross_stream_slices_ok(int Tn, int P);  // (below)

namespace {

constexpr int kTileBytes = 16 * 128;         // 16 keys x 64 elements x 2 bytes
constexpr int kStageBytes = 2 * kTileBytes;  // K tile + V tile
constexpr int kErrTimeout = 1;
constexpr int kPart = kD + 4;  // floats per query of a partial: acc[64], m, l, 2 pad (16-byte aligned records)

// A warp hands stages it has read back to the TMA: every lane's shared-memory reads of them (ldmatrix, generic proxy)
// are ordered before the copies that refill them (async proxy) by a proxy fence in each lane, then a warp barrier,
// after which one lane issues the copies. Without the fence nothing orders the two proxies: the compiler may sink a
// fragment load below the copy's issue, and the copy then overwrites the tile before the load reads it (measured at
// 16 queries per window, 20 heads x 1500 frames: without the fence most launches had one (window, head) wrong, with
// it none of 40).
__device__ __forceinline__ void release_stages() {
  fence_proxy_async_smem();
  __syncwarp();
}

// Launch shapes: streaming warps per CTA (plus the service warp) x ring stages per warp x CTAs per SM. Shared
// memory: warps * stages * 4 KB per CTA. Small problems (under 24 blocks per warp with shape 2) take shape 2,
// 5 (+1) warps x 5 stages x 2 CTAs: 10 streaming warps and 200 KB of ring per SM; larger ones shape 5, 3 (+1) warps
// x 8 stages x 2 CTAs: fewer, longer ranges (fewer partials per (window, head)) with the same bytes in flight.
// Measured (us per launch / per config step): 8 windows 20.1 (shape 2) vs 20.6 (shape 5); 32 windows 49.5 vs 48.5,
// step 1919 vs 1911; 64 windows step 4680 vs 4567. 5 x 9 x 1 CTA and 8 x 6 x 1 CTA were slower at both sizes.
struct Shape {
  int warps, stages;
  bool pair;  // two 16-key blocks per step of the online softmax
  int ctas;   // CTAs per SM
};
constexpr Shape kShapes[] = {{11, 4, false, 1}, {11, 4, true, 1}, {5, 5, true, 2},
                             {5, 4, true, 2},   {11, 5, true, 1}, {3, 8, true, 2}};

constexpr int smem_bytes(int warps, int stages) {
  return warps * stages * kStageBytes + warps * stages * 8 + warps * 24 + 1024;
}

struct StreamArgs {
  const void *q;
  void *y;
  float *part;
  int *counters;
  int *err;
  float *slices_out;  // slice mode: the reference's partials [W, H, P, S, D + 2] instead of y (null: fused output)
  int P, chunk;       // key slices per (window, head) and keys per slice (fused: 1 and Tn)
  int W, S, H, Tn, QG, bpu;
  long long total;
  long long per_warp;
  int max_slots;
  float scale;
  uint32_t polls;  // bound of every wait (wt_set_wait_limit)
  int withhold;    // test hook: no copy for the first stage of warp 0 of CTA 0 (wt_set_test_withhold_stage)
};

__host__ __device__ inline long long first_warp(long long u, int bpu, long long per_warp) {
  return u * bpu / per_warp;
}
__host__ __device__ inline long long last_warp(long long u, int bpu, long long per_warp) {
  return ((u + 1) * bpu - 1) / per_warp;
}

// A unit u = ((window * H + head) * P + slice) * QG + query group.
struct UnitPos {
  int w, h, sl, qg;
};
__device__ __forceinline__ UnitPos unit_pos(const StreamArgs &a, long long u) {
  UnitPos p;
  p.qg = static_cast<int>(u % a.QG);
  const long long r = u / a.QG;
  p.sl = static_cast<int>(r % a.P);
  const int wh = static_cast<int>(r / a.P);
  p.w = wh / a.H;
  p.h = wh - p.w * a.H;
  return p;
}

// Slice mode: one query's slice partial (unnormalised acc[64], running maximum m in log2 units, sum of exponentials l)
// into the reference's part layout [W, H, P, S, D + 2].
__device__ __forceinline__ float *slice_record(const StreamArgs &a, const UnitPos &p, int qi) {
  return a.slices_out + ((((static_cast<size_t>(p.w) * a.H + p.h) * a.P + p.sl) * a.S + qi) * (kD + 2));
}

template <int NT>
__device__ __forceinline__ void reset_state(State<NT> &st) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    st.m[nt][0] = st.m[nt][1] = kNegInf;
    st.l[nt][0] = st.l[nt][1] = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) st.o[nt][i][j] = 0.f;
  }
}

// The warp's partial for unit u -> workspace (plain stores: nothing waits for them here; the count that publishes
// them comes later, behind a fence -- see publish() and serve_requests()).
template <int NT>
__device__ __forceinline__ void write_record(State<NT> &st, float *dst, int lane);
template <typename T, int NT>
__device__ void combine_records(const StreamArgs &a, const float *base, int nslots, const UnitPos &up, int lane);

template <int NT>
__device__ __forceinline__ void store_partial(State<NT> &st, const StreamArgs &a, long long u, long long gw,
                                              int lane) {
  const long long fw = first_warp(u, a.bpu, a.per_warp);
  const int slot = static_cast<int>(gw - fw);
  write_record<NT>(st, a.part + (static_cast<size_t>(u) * a.max_slots + slot) * (NT * 8) * kPart, lane);
}

// A warp's online-softmax state -> one record per query of NT * 8 (acc[64], m, l, 2 pad: 16-byte aligned), its
// row sums first reduced over the lanes that hold them.
template <int NT>
__device__ __forceinline__ void write_record(State<NT> &st, float *dst, int lane) {
  const int g = lane >> 2, c = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) st.l[nt][j] += __shfl_xor_sync(0xffffffffu, st.l[nt][j], o);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float *rq = dst + (nt * 8 + 2 * c + j) * kPart;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        rq[16 * i + g] = st.o[nt][i][j];
        rq[16 * i + g + 8] = st.o[nt][i][j + 2];
      }
      if (g == 0) {
        rq[kD] = st.m[nt][j];
        rq[kD + 1] = st.l[nt][j];
      }
    }
}

// The warp's block count for unit u added to the unit's counter by one acquire-release atomic (lane 0, after a warp
// barrier): its release side orders the partial every lane of this warp stored before it, its acquire side the
// other warps' partials before whatever this warp reads next (combine_unit). Returns, in lane 0, whether this warp
// completed the unit.
__device__ __forceinline__ bool publish(const StreamArgs &a, long long u, int nblk, int lane) {
  __syncwarp();
  int old = 0;
  if (lane == 0)
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(a.counters + u), "r"(nblk) : "memory");
  return old + nblk == a.bpu;
}

// A unit this warp attended whole: its output straight from the registers (acc / l per query; the running maximum is
// common to both), no partial and no counter.
template <typename T, int NT>
__device__ __forceinline__ void finalize_unit(State<NT> &st, const StreamArgs &a, long long u, int lane) {
  const int g = lane >> 2, c = lane & 3;
  const UnitPos p = unit_pos(a, u);
  const int w = p.w, h = p.h, qg = p.qg;
  const size_t HD = static_cast<size_t>(a.H) * kD;
  T *y = static_cast<T *>(a.y);
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float l = st.l[nt][j];
#pragma unroll
      for (int o = 4; o < 32; o <<= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
      const int qi = qg * NT * 8 + nt * 8 + 2 * c + j;
      if (qi < a.S && a.slices_out != nullptr) {  // slice mode: the slice's unnormalised partial
        float *rec = slice_record(a, p, qi);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          rec[16 * i + g] = st.o[nt][i][j];
          rec[16 * i + g + 8] = st.o[nt][i][j + 2];
        }
        if (g == 0) {
          rec[kD] = st.m[nt][j];
          rec[kD + 1] = l;
        }
      } else if (qi < a.S) {
        const float inv = 1.f / l;
        T *yr = y + (static_cast<size_t>(w) * a.S + qi) * HD + static_cast<size_t>(h) * kD;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          yr[16 * i + g] = Elem<T>::from_float(st.o[nt][i][j] * inv);
          yr[16 * i + g + 8] = Elem<T>::from_float(st.o[nt][i][j + 2] * inv);
        }
      }
    }
}

// The warp that completed unit u: every partial of u -> the output (then the counter back to zero). Each lane owns
// (query, 8-dim chunk) items; for a pass of up to kCombineSlots partials it issues every load first (one L2 round
// trip), then folds them into a running (top, den, num) -- the reference's combine (attn_plugin.py:182-194), merged
// pass by pass.
constexpr int kCombineSlots = 4;
template <typename T, int NT>
__device__ void combine_records(const StreamArgs &a, const float *base, int nslots, const UnitPos &up, int lane);

template <typename T, int NT>
__device__ void combine_unit(const StreamArgs &a, long long u, int lane) {
  __syncwarp();  // (after lane 0's acquire-release count: every lane's loads below are ordered after it)
  const long long fw = first_warp(u, a.bpu, a.per_warp);
  const int nslots = static_cast<int>(last_warp(u, a.bpu, a.per_warp) - fw + 1);
  combine_records<T, NT>(a, a.part + static_cast<size_t>(u) * a.max_slots * (NT * 8) * kPart, nslots,
                         unit_pos(a, u), lane);
  if (lane == 0) a.counters[u] = 0;  // left zeroed for the next launch
}

// `nslots` records of one (window, head, query group) at `base` -> the output (or, slice mode, the slice's part).
template <typename T, int NT>
__device__ void combine_records(const StreamArgs &a, const float *base, int nslots, const UnitPos &up, int lane) {
  const int w = up.w, h = up.h, qg = up.qg;
  const int q0 = qg * NT * 8;
  const int nq = min(NT * 8, a.S - q0);
  const size_t HD = static_cast<size_t>(a.H) * kD;
  T *y = static_cast<T *>(a.y);
  constexpr int kItems = NT * 8 * (kD / 8) / 32;  // items per lane (NT * 2)
#pragma unroll
  for (int it0 = 0; it0 < kItems; it0 += 2) {
    float top[2], den[2], num[2][8];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      top[k] = kNegInf;
      den[k] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) num[k][i] = 0.f;
    }
    for (int s0 = 0; s0 < nslots; s0 += kCombineSlots) {
      float ml[2][kCombineSlots][2];
      float4 av[2][kCombineSlots][2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int idx = lane + 32 * (it0 + k), qq = idx >> 3, d8 = idx & 7;
#pragma unroll
        for (int s2 = 0; s2 < kCombineSlots; ++s2) {
          if (qq < nq && s0 + s2 < nslots) {
            const float *ps = base + ((s0 + s2) * NT * 8 + qq) * kPart;
            const float2 v = __ldcg(reinterpret_cast<const float2 *>(ps + kD));
            ml[k][s2][0] = v.x;
            ml[k][s2][1] = v.y;
            av[k][s2][0] = __ldcg(reinterpret_cast<const float4 *>(ps + 8 * d8));
            av[k][s2][1] = __ldcg(reinterpret_cast<const float4 *>(ps + 8 * d8 + 4));
          } else {
            ml[k][s2][0] = kNegInf;
            ml[k][s2][1] = 0.f;
            av[k][s2][0] = av[k][s2][1] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        float nt_top = top[k];
#pragma unroll
        for (int s2 = 0; s2 < kCombineSlots; ++s2) nt_top = fmaxf(nt_top, ml[k][s2][0]);
        if (nt_top == kNegInf) continue;  // (no keys yet: nothing to fold)
        const float f = top[k] == kNegInf ? 0.f : ex2(top[k] - nt_top);
        den[k] *= f;
#pragma unroll
        for (int i = 0; i < 8; ++i) num[k][i] *= f;
        top[k] = nt_top;
#pragma unroll
        for (int s2 = 0; s2 < kCombineSlots; ++s2) {
          const float wgt = ml[k][s2][0] == kNegInf ? 0.f : ex2(ml[k][s2][0] - nt_top);
          den[k] = fmaf(wgt, ml[k][s2][1], den[k]);
          const float4 x = av[k][s2][0], z = av[k][s2][1];
          num[k][0] = fmaf(wgt, x.x, num[k][0]);
          num[k][1] = fmaf(wgt, x.y, num[k][1]);
          num[k][2] = fmaf(wgt, x.z, num[k][2]);
          num[k][3] = fmaf(wgt, x.w, num[k][3]);
          num[k][4] = fmaf(wgt, z.x, num[k][4]);
          num[k][5] = fmaf(wgt, z.y, num[k][5]);
          num[k][6] = fmaf(wgt, z.z, num[k][6]);
          num[k][7] = fmaf(wgt, z.w, num[k][7]);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int idx = lane + 32 * (it0 + k), qq = idx >> 3, d8 = idx & 7;
      if (qq < nq && a.slices_out != nullptr) {  // slice mode: the combined, still unnormalised partial
        float *rec = slice_record(a, up, q0 + qq);  // (records of D + 2 floats: 8-byte aligned)
#pragma unroll
        for (int i = 0; i < 8; i += 2)
          *reinterpret_cast<float2 *>(rec + 8 * d8 + i) = make_float2(num[k][i], num[k][i + 1]);
        if (d8 == 0) {
          rec[kD] = top[k];
          rec[kD + 1] = den[k];
        }
      } else if (qq < nq) {
        const float inv = 1.f / den[k];
#pragma unroll
        for (int i = 0; i < 8; ++i) num[k][i] *= inv;
        *reinterpret_cast<uint4 *>(y + (static_cast<size_t>(w) * a.S + q0 + qq) * HD + static_cast<size_t>(h) * kD +
                                   8 * d8) = pack8<T>(num[k]);
      }
    }
  }
}

// The CTA's service warp: lane i waits for streaming warp i's request (its first unit's partial stored, or none),
// then adds the warp's block count to the unit's counter with an acquire-release atomic -- its release side covers
// the streaming warp's stores, ordered before its mbarrier arrival, which this lane's wait acquires. Units it
// completes it combines itself. The polls are bounded: on a timeout the error word gets a code and the warp returns.
template <typename T, int NT, int kStreamWarps>
__device__ void serve_requests(const StreamArgs &a, uint64_t *req_bar, const long long *req_u, const int *req_n,
                               int lane) {
  bool waiting = lane < kStreamWarps;
  for (uint32_t it = 0; it < a.polls; ++it) {
    long long u = -1;
    bool completed = false;
    if (waiting && mbar_try_wait(&req_bar[lane], 0)) {
      waiting = false;
      u = req_u[lane];
      if (u >= 0) {
        const int nb = req_n[lane];
        int old = 0;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(a.counters + u), "r"(nb) : "memory");
        completed = old + nb == a.bpu;
      }
    }
    for (unsigned m = __ballot_sync(0xffffffffu, completed); m; m &= m - 1)
      combine_unit<T, NT>(a, __shfl_sync(0xffffffffu, u, __ffs(m) - 1), lane);
    if (!__any_sync(0xffffffffu, waiting)) return;
    if (it > 64) __nanosleep(64);
  }
  if (lane == 0) atomicExch(a.err, kErrTimeout);
}

template <typename T, int NT, int kStreamWarps, int kStreamStages, bool kPair, int kCtas>
__global__ void __launch_bounds__((kStreamWarps + 1) * 32, kCtas)
    cross_stream_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const StreamArgs a) {
  constexpr int kWarpRing = kStreamStages * kStageBytes;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  uint64_t *req_bar = reinterpret_cast<uint64_t *>(smem + kStreamWarps * kWarpRing) + kStreamWarps * kStreamStages;
  long long *req_u = reinterpret_cast<long long *>(req_bar + kStreamWarps);
  int *req_n = reinterpret_cast<int *>(req_u + kStreamWarps);
  if (warp == kStreamWarps) {  // the service warp
    if (lane < kStreamWarps) mbar_init(&req_bar[lane], 1);
    fence_mbar_init();
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();
    serve_requests<T, NT, kStreamWarps>(a, req_bar, req_u, req_n, lane);
    return;
  }
  unsigned char *ring = smem + warp * kWarpRing;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kStreamWarps * kWarpRing) + warp * kStreamStages;
  const long long gw = static_cast<long long>(blockIdx.x) * kStreamWarps + warp;
  const long long beg = gw * a.per_warp;
  const long long end = min(beg + a.per_warp, a.total);
  if (lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
#pragma unroll
    for (int s = 0; s < kStreamStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncthreads();  // (the service warp's request barriers are initialised)
  const int n = beg < end ? static_cast<int>(end - beg) : 0;

  // the range's position as (window-head, query group, block), advanced without divisions
  const long long u0 = n ? beg / a.bpu : 0;
  int i_qg = static_cast<int>(u0 % a.QG), i_sl = static_cast<int>((u0 / a.QG) % a.P);
  int i_wh = static_cast<int>(u0 / a.QG / a.P);
  int i_b = static_cast<int>(beg - u0 * a.bpu);
  int issued = 0;
  // (the bounded-wait test hook: warp 0 of CTA 0 issues nothing for its first stage, whose wait then runs out)
  const bool withhold = a.withhold && gw == 0;
  auto issue_next = [&]() {  // lane 0: the next block of the range into its stage
    const int s = issued % kStreamStages;
    unsigned char *dst = ring + s * kStageBytes;
    const int row = i_wh * a.Tn + i_sl * a.chunk + i_b * 16;
    if (!(withhold && issued == 0)) {
      mbar_arrive_expect_tx(&bars[s], kStageBytes);
      tma_load_2d(dst, &kmap, 0, row, &bars[s]);
      tma_load_2d(dst + kTileBytes, &vmap, 0, row, &bars[s]);
    }
    ++issued;
    if (++i_b == a.bpu) {
      i_b = 0;
      if (++i_qg == a.QG) {
        i_qg = 0;
        if (++i_sl == a.P) {
          i_sl = 0;
          ++i_wh;
        }
      }
    }
  };
  if (lane == 0)
    while (issued < min(n, kStreamStages)) issue_next();
  // (everything above reads only the cross keys/values, which the kernel launched just before this one does not
  // write; the queries, the workspace and the output wait for it)
  pdl_wait();
  // the next kernel may launch now: it reads nothing this kernel writes before its own wait, which waits for
  // this kernel to complete
  pdl_launch_dependents();

  const T *q = static_cast<const T *>(a.q);
  const size_t HD = static_cast<size_t>(a.H) * kD;
  uint32_t qf[NT][8], qn[NT][8];  // this unit's query fragments, and the next unit's, loaded one unit ahead
  State<NT> st;
  long long cur = -1;
  int nblk = 0;
  int stop = -1;  // the block whose wait timed out: nothing is consumed or issued from it on
  // Only a range's first unit (when it began in an earlier warp's range) and its last one (when it goes on into the
  // next warp's range) are shared with other warps: they go through partials and the units' counters; a unit wholly
  // inside the range goes straight to the output from registers. The first unit, when the range goes on past it, is
  // handed to the CTA's service warp once its partial is stored: an mbarrier arrival (a CTA-scope release) instead of
  // the GPU-scope fence a count needs, which would stall this warp -- with its loads in flight -- for about as long
  // as eight blocks take to stream (measured). The last unit is counted by this warp at the end of its range.
  const bool first_shared = beg % a.bpu != 0;
  bool handed = !(n > 0 && first_shared && beg + n > (u0 + 1) * a.bpu);  // the service warp's request is posted
  if (handed && lane == 0) {  // no such unit: say so
    req_u[warp] = -1;
    mbar_arrive(&req_bar[warp]);
  }
  int c_qg = static_cast<int>(u0 % a.QG), c_sl = static_cast<int>((u0 / a.QG) % a.P);
  int c_wh = static_cast<int>(u0 / a.QG / a.P);
  int c_b = static_cast<int>(beg - u0 * a.bpu);
  long long c_u = u0;
  for (int j = 0; j < n;) {
    if (c_u != cur) {
      if (cur >= 0) {
        if (cur == u0 && first_shared) {
          store_partial<NT>(st, a, cur, gw, lane);
          __syncwarp();  // (every lane's stores before lane 0's arrival)
          if (lane == 0) {
            req_u[warp] = cur;
            req_n[warp] = nblk;
            mbar_arrive(&req_bar[warp]);
          }
          handed = true;
        } else {
          finalize_unit<T, NT>(st, a, cur, lane);
        }
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int i = 0; i < 8; ++i) qf[nt][i] = qn[nt][i];
      } else {
        const int w = c_wh / a.H, h = c_wh - w * a.H;
        load_q_std<T, NT>(qf, q + static_cast<size_t>(w) * a.S * HD + static_cast<size_t>(h) * kD, HD,
                          c_qg * NT * 8, a.S, g, c);
      }
      cur = c_u;
      nblk = 0;
      reset_state<NT>(st);
      // the next unit's queries, needed only after this unit's blocks of the range
      int n_wh = c_wh, n_qg = c_qg + 1;
      if (n_qg == a.QG) {
        n_qg = 0;
        if (c_sl + 1 == a.P) ++n_wh;
      }
      if (n_wh < a.W * a.H) {
        const int w = n_wh / a.H, h = n_wh - w * a.H;
        load_q_std<T, NT>(qn, q + static_cast<size_t>(w) * a.S * HD + static_cast<size_t>(h) * kD, HD,
                          n_qg * NT * 8, a.S, g, c);
      }
    }
    // two blocks at once when the range's next block belongs to the same (window, head)
    const bool pair = kPair && j + 1 < n && c_b + 1 < a.bpu;
    const int s0 = j % kStreamStages, s1 = (j + 1) % kStreamStages;
    // a wait that runs out (in any lane: the warp decides together) stops the range here, error word set: the stage
    // is neither read nor refilled, so every stage keeps at most one copy outstanding and the drain below can wait
    // for each by its own phase
    bool ok = mbar_wait_bounded(&bars[s0], static_cast<uint32_t>((j / kStreamStages) & 1), a.err, kErrTimeout, a.polls);
    if (pair && ok)
      ok = mbar_wait_bounded(&bars[s1], static_cast<uint32_t>(((j + 1) / kStreamStages) & 1), a.err, kErrTimeout,
                             a.polls);
    if (!__all_sync(0xffffffffu, ok)) {
      stop = j;
      break;
    }
    uint32_t ka[4][4], va[4][4];
    smem_frags(ka, va, ring + s0 * kStageBytes, ring + s0 * kStageBytes + kTileBytes, lane);
    const int k0 = c_b * 16;
    const int klen = min(a.Tn - c_sl * a.chunk, a.chunk);  // keys of the unit's slice (fused: all Tn)
    const int used = pair ? 2 : 1;
    if (pair) {
      uint32_t kb[4][4], vb[4][4];
      smem_frags(kb, vb, ring + s1 * kStageBytes, ring + s1 * kStageBytes + kTileBytes, lane);
      // refill both stages now, so every stage of the ring is in flight while this warp computes: each lane's
      // reads of them ordered before the copies (release_stages), then one lane issues
      release_stages();
      if (lane == 0)
        for (int u = 0; u < used && issued < n; ++u) issue_next();
      const bool ok[2][2] = {{k0 + g < klen, k0 + g + 8 < klen}, {k0 + 16 + g < klen, k0 + 24 + g < klen}};
      attend_block2<T, NT>(st, ka, va, kb, vb, qf, ok, a.scale);
    } else {
      release_stages();
      if (lane == 0 && issued < n) issue_next();
      attend_block<T, NT>(st, ka, va, qf, k0 + g < klen, k0 + g + 8 < klen, a.scale);
    }
    nblk += used;
    j += used;
    c_b += used;
    if (c_b == a.bpu) {
      c_b = 0;
      ++c_u;
      if (++c_qg == a.QG) {
        c_qg = 0;
        if (++c_sl == a.P) {
          c_sl = 0;
          ++c_wh;
        }
      }
    }
  }
  if (stop >= 0) {
    // a timed-out wait: before the shared memory goes away, wait (bounded, again) for every copy still outstanding
    // -- blocks stop .. issued - 1, at most one per stage -- and leave the range's units unfinished (the output is
    // invalid and the error word says so; the workspace must be zeroed again before its next use)
    const int iss = __shfl_sync(0xffffffffu, issued, 0);
    for (int jj = stop; jj < iss; ++jj)
      if (!(withhold && jj == 0))
        mbar_wait_bounded(&bars[jj % kStreamStages], static_cast<uint32_t>((jj / kStreamStages) & 1), nullptr, 0,
                          a.polls);
    if (!handed && lane == 0) {  // (the service warp is told there is nothing to count)
      req_u[warp] = -1;
      mbar_arrive(&req_bar[warp]);
    }
    return;
  }
  // the last unit: shared if it began before the range or goes on after it (the loop did not step past its last block)
  const bool last_shared = cur >= 0 && ((cur == u0 && first_shared) || c_u == cur);
  if (cur >= 0) {
    if (last_shared)
      store_partial<NT>(st, a, cur, gw, lane);
    else
      finalize_unit<T, NT>(st, a, cur, lane);
  }
  if (last_shared) {
    if (__shfl_sync(0xffffffffu, publish(a, cur, nblk, lane) ? 1 : 0, 0)) combine_unit<T, NT>(a, cur, lane);
  }
}

// Fused attention of few windows, one CTA per (window, head): its kWinSlices warps each stream one key slice of the
// window's frames through their own TMA ring (16-key blocks, two at a time), and the slices' online-softmax states
// meet in shared memory after a CTA barrier, where 8 threads per query combine them into the output. No partial
// leaves the SM and no counter is taken: the tail after the last block is a few hundred cycles (the stream-K and
// slice-unit kernels end with a partial's stores, a GPU-scope count and an L2 round trip per combined slice). With
// programmatic dependent launch the first stages' loads go out before the wait for the preceding kernel.
// Shapes (slices = warps per CTA, ring stages per warp, CTAs per SM: shared memory allows no more). The launch takes
// the shape whose whole waves of CTAs waste the fewest unit slots (window_shape_for), as measured on B200 per launch
// chained (same kernel back to back) at 8 / 16 / 24 / 32 / 64 windows of 20 heads x 1500 frames: (8, 3, 2) 16.6 /
// 30.4 / 35.0 / 48.1 / 81.1 us; (4, 4, 3) 17.4 / 24.8 / 43.2 / 45.3 / 78.5; (4, 3, 4) 18.6 / 24.8 / 33.3 / 52.0 / 84.8
// -- a launch whose last wave is a small fraction of the resident CTAs pays for it (24 windows on (4, 4, 3), 32 on
// (4, 3, 4)); the decode step at 32 windows (config 3) 2.033 -> 1.913 ms on (4, 4, 3), at 16 windows (config 4)
// 1.350 -> 1.244 ms, at 8 windows (config 2) 0.579 -> 0.647 ms (so (8, 3, 2) there). Also measured, slower at every
// size: (16, 2, 1), (16, 3, 1), (12, 3, 1), (6, 4, 2), (4, 6, 2), (5, 5, 2), (6, 3, 2), and 3 CTAs of 6-12 warps
// (registers spill). WT_CROSS_WIN_SHAPE (a tuning knob) forces one.
struct WinShape {
  int slices, stages, ctas;
};
constexpr WinShape kWinShapes[] = {{8, 3, 2}, {16, 2, 1}, {4, 4, 3}, {4, 3, 4}};
constexpr int kNumWinShapes = static_cast<int>(sizeof(kWinShapes) / sizeof(kWinShapes[0]));
constexpr int win_smem(int slices, int stages) { return slices * stages * kStageBytes + slices * stages * 8 + 1024; }

template <typename T, int kWinSlices, int kWinStages, int kWinCtas>
__global__ void __launch_bounds__(kWinSlices * 32, kWinCtas)
    cross_window_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                        const T *__restrict__ q, T *__restrict__ y, int *err, int S, int H, int Tn, int chunk,
                        float scale, uint32_t polls, int withhold) {
  constexpr int kWinRing = kWinStages * kStageBytes;
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem =
      reinterpret_cast<unsigned char *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int wh = blockIdx.x, w = wh / H, h = wh - (wh / H) * H;
  unsigned char *ring = smem + warp * kWinRing;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kWinSlices * kWinRing) + warp * kWinStages;
  const int k_lo = warp * chunk;
  const int klen = max(0, min(Tn - k_lo, chunk));  // keys of this warp's slice
  const int nblk = (klen + 15) / 16;
  if (lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
#pragma unroll
    for (int s = 0; s < kWinStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const int row0 = wh * Tn + k_lo;
  // (the bounded-wait test hook: warp 0 of CTA 0 issues nothing for its first block, whose wait then runs out)
  const bool hold = withhold && wh == 0 && warp == 0;
  auto issue = [&](int b) {  // lane 0: block b of the slice into its stage
    const int s = b % kWinStages;
    unsigned char *dst = ring + s * kStageBytes;
    if (hold && b == 0) return;
    mbar_arrive_expect_tx(&bars[s], kStageBytes);
    tma_load_2d(dst, &kmap, 0, row0 + b * 16, &bars[s]);
    tma_load_2d(dst + kTileBytes, &vmap, 0, row0 + b * 16, &bars[s]);
  };
  if (lane == 0)
    for (int b = 0; b < min(nblk, kWinStages); ++b) issue(b);
  // (the cross keys/values are not the preceding kernel's output; the queries and the output wait for it)
  pdl_wait();
  pdl_launch_dependents();

  const size_t HD = static_cast<size_t>(H) * kD;
  uint32_t qf[1][8];
  load_q_std<T, 1>(qf, q + static_cast<size_t>(w) * S * HD + static_cast<size_t>(h) * kD, HD, 0, S, g, c);
  State<1> st;
  reset_state<1>(st);
  int stop = -1;  // the block whose wait timed out: nothing is consumed or issued from it on
  for (int j = 0; j < nblk;) {
    const bool pair = j + 1 < nblk;
    const int s0 = j % kWinStages, s1 = (j + 1) % kWinStages;
    // a wait that runs out (in any lane: the warp decides together) stops the slice here, error word set: the
    // stage is neither read nor refilled, so every stage keeps at most one copy outstanding for the drain below
    bool ok = mbar_wait_bounded(&bars[s0], static_cast<uint32_t>((j / kWinStages) & 1), err, kErrTimeout, polls);
    if (pair && ok)
      ok = mbar_wait_bounded(&bars[s1], static_cast<uint32_t>(((j + 1) / kWinStages) & 1), err, kErrTimeout, polls);
    if (!__all_sync(0xffffffffu, ok)) {
      stop = j;
      break;
    }
    uint32_t ka[4][4], va[4][4];
    smem_frags(ka, va, ring + s0 * kStageBytes, ring + s0 * kStageBytes + kTileBytes, lane);
    const int k0 = j * 16;
    if (pair) {
      uint32_t kb[4][4], vb[4][4];
      smem_frags(kb, vb, ring + s1 * kStageBytes, ring + s1 * kStageBytes + kTileBytes, lane);
      release_stages();
      if (lane == 0) {  // refill both stages (every lane's reads of them are ordered before the copies)
        if (j + kWinStages < nblk) issue(j + kWinStages);
        if (j + 1 + kWinStages < nblk) issue(j + 1 + kWinStages);
      }
      const bool ok[2][2] = {{k0 + g < klen, k0 + g + 8 < klen}, {k0 + 16 + g < klen, k0 + 24 + g < klen}};
      attend_block2<T, 1>(st, ka, va, kb, vb, qf, ok, scale);
      j += 2;
    } else {
      release_stages();
      if (lane == 0 && j + kWinStages < nblk) issue(j + kWinStages);
      attend_block<T, 1>(st, ka, va, qf, k0 + g < klen, k0 + g + 8 < klen, scale);
      j += 1;
    }
  }
  if (stop >= 0) {
    // a timed-out wait: wait (bounded, again) for every copy still outstanding -- blocks stop .. stop + stages - 1,
    // at most one per stage -- so that no copy lands in the ring after it is reused below or the CTA has exited
    // (this slice's record is left out: the output is invalid and the error word says so)
    for (int jj = stop; jj < min(nblk, stop + kWinStages); ++jj)
      if (!(hold && jj == 0))
        mbar_wait_bounded(&bars[jj % kWinStages], static_cast<uint32_t>((jj / kWinStages) & 1), nullptr, 0, polls);
  }
  // this slice's state (acc, m, l per query) over the start of its ring: every stage has been consumed
  __syncwarp();
  float *rec = reinterpret_cast<float *>(ring);
  if (stop < 0) write_record<1>(st, rec, lane);
  __syncthreads();
  // the slices' states -> the output: thread t takes query t / 8, head dims 8 (t % 8) .. + 7 (attn_plugin.py:182-194)
  for (int t = threadIdx.x; t < S * 8; t += blockDim.x) {
    const int qq = t >> 3, d8 = t & 7;
    float top = kNegInf;
#pragma unroll
    for (int sl = 0; sl < kWinSlices; ++sl) {
      const float *r = reinterpret_cast<const float *>(smem + sl * kWinRing) + qq * kPart;
      top = fmaxf(top, r[kD]);
    }
    float den = 0.f, num[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int sl = 0; sl < kWinSlices; ++sl) {
      const float *r = reinterpret_cast<const float *>(smem + sl * kWinRing) + qq * kPart;
      const float ms = r[kD];
      const float wgt = ms == kNegInf ? 0.f : ex2(ms - top);
      den = fmaf(wgt, r[kD + 1], den);
      const float4 x = *reinterpret_cast<const float4 *>(r + 8 * d8), z = *reinterpret_cast<const float4 *>(r + 8 * d8 + 4);
      num[0] = fmaf(wgt, x.x, num[0]);
      num[1] = fmaf(wgt, x.y, num[1]);
      num[2] = fmaf(wgt, x.z, num[2]);
      num[3] = fmaf(wgt, x.w, num[3]);
      num[4] = fmaf(wgt, z.x, num[4]);
      num[5] = fmaf(wgt, z.y, num[5]);
      num[6] = fmaf(wgt, z.z, num[6]);
      num[7] = fmaf(wgt, z.w, num[7]);
    }
    const float inv = 1.f / den;
#pragma unroll
    for (int i = 0; i < 8; ++i) num[i] *= inv;
    *reinterpret_cast<uint4 *>(y + (static_cast<size_t>(w) * S + qq) * HD + static_cast<size_t>(h) * kD + 8 * d8) =
        pack8<T>(num);
  }
}

// The SM count the plan is sized for (148 on a B200 if the device cannot be queried: the launch then reports the
// device's own error).
int sm_count() {
  const int n = device_sm_count();
  return n > 0 ? n : 148;
}

// A launch shape forced by the WT_CROSS_SHAPE environment variable (a tuning knob), or -1.
int forced_shape() {
  static const int idx = [] {  // (read once; a function-local static initialises thread-safely)
    const char *e = getenv("WT_CROSS_SHAPE");
    const int v = e ? atoi(e) : -1;
    return (v >= 0 && v < static_cast<int>(sizeof(kShapes) / sizeof(kShapes[0]))) ? v : -1;
  }();
  return idx;
}

struct StreamPlan {
  int nt, qgs, bpu, max_slots, grid, shape, slices, chunk;
  long long units, total, per_warp;
  size_t counters_off, part_off, bytes;
};

// The one-CTA-per-(window, head) kernel takes the fused attention when a window has at most 8 queries (one query
// tile) and every 16-key block of the chosen shape's slices holds a key; the stream-K kernel the rest. Measured per launch, chained
// as in the step (stream-K -> this kernel): 8 windows 14.3 -> 13.3 us, 32 windows 44.2 -> 43.7 us, 64 windows 91.6 ->
// 78.1 us (the CTAs' dynamic scheduling leaves a smaller tail than the stream-K ranges' unit-boundary combines).
// WT_CROSS_WINDOW=0 (a tuning knob) turns it off.
int forced_window_shape() {
  static const int idx = [] {  // (read once; a function-local static initialises thread-safely)
    const char *e = getenv("WT_CROSS_WIN_SHAPE");
    const int v = e ? atoi(e) : -1;
    return (v >= 0 && v < kNumWinShapes) ? v : -1;
  }();
  return idx;
}

// The window kernel's shape for W x H (window, head) units over Tn frames, or -1 if none fits (some 16-key block of a
// slice would hold no key): among (4, 4, 3), (4, 3, 4) and (8, 3, 2), in that order of preference on ties, the one
// whose whole waves -- ceil(units / resident CTAs) x resident CTAs -- leave the fewest slots idle.
int window_shape_for(int W, int H, int Tn) {
  const int forced = forced_window_shape();
  if (forced >= 0) return cross_stream_slices_ok(Tn, kWinShapes[forced].slices) ? forced : -1;
  const long long units = static_cast<long long>(W) * H;
  int best = -1;
  long long best_slots = 0;
  for (const int i : {2, 3, 0}) {
    if (!cross_stream_slices_ok(Tn, kWinShapes[i].slices)) continue;
    const long long resident = static_cast<long long>(sm_count()) * kWinShapes[i].ctas;
    const long long slots = (units + resident - 1) / resident * resident;
    if (best < 0 || slots < best_slots) {
      best = i;
      best_slots = slots;
    }
  }
  return best;
}

bool window_kernel_ok(int W, int S, int H, int Tn) {
  static const int off = [] {  // (read once; a function-local static initialises thread-safely)
    const char *e = getenv("WT_CROSS_WINDOW");
    return (e != nullptr && atoi(e) == 0) ? 1 : 0;
  }();
  return !off && W > 0 && H > 0 && S <= 8 && window_shape_for(W, H, Tn) >= 0;
}

template <typename T, int SL, int ST, int CT>
int launch_window_shape(const CUtensorMap &km, const CUtensorMap &vm, const void *q, void *y, int *err, int W,
                        int S, int H, int Tn, float scale, void *stream) {
  constexpr int smem = win_smem(SL, ST);
  const int st = opt_in_smem<cross_window_kernel<T, SL, ST, CT>>(smem, "cross_attn");
  if (st != WT_OK) return st;
  const int chunk = (Tn + SL - 1) / SL;
  return launch("cross_attn", cross_window_kernel<T, SL, ST, CT>, dim3(W * H), dim3(SL * 32), smem, stream, km, vm,
                static_cast<const T *>(q), static_cast<T *>(y), err, S, H, Tn, chunk, scale, wait_limit(),
                test_withhold_stage());
}

template <typename T>
int launch_window(const CUtensorMap &km, const CUtensorMap &vm, const void *q, void *y, int *err, int W, int S,
                  int H, int Tn, float scale, void *stream) {
  switch (window_shape_for(W, H, Tn)) {
#define WT_WIN_CASE(i)                                                                                           \
  case i:                                                                                                        \
    return launch_window_shape<T, kWinShapes[i].slices, kWinShapes[i].stages, kWinShapes[i].ctas>(km, vm, q, y, err, \
                                                                                                 W, S, H, Tn, scale, \
                                                                                                 stream);
    WT_WIN_CASE(1)
    WT_WIN_CASE(2)
    WT_WIN_CASE(3)
#undef WT_WIN_CASE
    default:
      return launch_window_shape<T, kWinShapes[0].slices, kWinShapes[0].stages, kWinShapes[0].ctas>(km, vm, q, y, err,
                                                                                                    W, S, H, Tn, scale,
                                                                                                    stream);
  }
}

// P = 0: the fused attention (a unit is a whole (window, head, query group)); P > 0: slice mode, P key slices of
// ceil(Tn / P) keys per (window, head), each its own unit, written as the reference's part.
StreamPlan plan_stream(int W, int S, int H, int Tn, int P) {
  StreamPlan p{};
  p.nt = (S + 7) / 8 > 4 ? 4 : (S + 7) / 8;
  p.qgs = (S + p.nt * 8 - 1) / (p.nt * 8);
  p.slices = P > 0 ? P : 1;
  p.chunk = P > 0 ? (Tn + P - 1) / P : Tn;
  p.bpu = (p.chunk + 15) / 16;
  p.units = static_cast<long long>(W) * H * p.slices * p.qgs;
  p.total = p.units * p.bpu;
  if (p.nt >= 2) {
    p.shape = 0;  // (more query tiles: one block per step keeps them in registers)
  } else if (forced_shape() >= 0) {
    p.shape = forced_shape();
  } else {
    // many blocks per warp: fewer, longer ranges -- 3 (+1) warps x 8 stages for whole (window, head) units, 5 (+1) x 4
    // in slice mode, whose 12-block units make more unit ends per range (measured at 32 windows: 44.8 us per launch
    // against 50.7 with 3 x 8)
    const long long w2 = static_cast<long long>(sm_count()) * kShapes[2].ctas * kShapes[2].warps;
    p.shape = (p.total + w2 - 1) / w2 >= 24 ? (P > 0 ? 3 : 5) : 2;
  }
  if (P > 0) {
    // slice mode: one warp per (window, head, slice) unit and as many CTAs as that takes -- the units are small and
    // equal, so the hardware's CTA scheduling balances them, and no range shares a unit (no partials, no counts):
    // after the GEMM before it, a persistent grid would pay its ramp and its unit-boundary combines every layer
    p.per_warp = p.bpu;
    const long long g = (p.units + kShapes[p.shape].warps - 1) / kShapes[p.shape].warps;
    p.grid = static_cast<int>(g < (1LL << 31) - 1 ? g : (1LL << 31) - 1);
  } else {
    p.grid = sm_count() * kShapes[p.shape].ctas;
    const long long warps = static_cast<long long>(p.grid) * kShapes[p.shape].warps;
    p.per_warp = (p.total + warps - 1) / warps;
  }
  p.max_slots = static_cast<int>((p.bpu + p.per_warp - 1) / p.per_warp + 1);
  p.counters_off = 256;  // [0, 256): the device error word
  p.part_off = p.counters_off + (static_cast<size_t>(p.units) * sizeof(int) + 255) / 256 * 256;
  // (slice mode shares no unit between warps: no partials)
  p.bytes = p.part_off + (P > 0 ? 0 : static_cast<size_t>(p.units) * p.max_slots * p.nt * 8 * kPart * sizeof(float));
  return p;
}

template <typename T, int NT, int WARPS, int STAGES, bool PAIR, int CTAS>
int launch_stream_shape(const CUtensorMap &km, const CUtensorMap &vm, const StreamArgs &a, int grid, void *stream) {
  constexpr int smem = smem_bytes(WARPS, STAGES);
  const int st = opt_in_smem<cross_stream_kernel<T, NT, WARPS, STAGES, PAIR, CTAS>>(smem, "cross_attn");
  if (st != WT_OK) return st;
  return launch("cross_attn", cross_stream_kernel<T, NT, WARPS, STAGES, PAIR, CTAS>, dim3(grid), dim3((WARPS + 1) * 32), smem,
                stream, km, vm, a);
}

template <typename T, int NT>
int launch_stream_nt(const CUtensorMap &km, const CUtensorMap &vm, const StreamArgs &a, int grid, int shape,
                     void *stream) {
  if constexpr (NT >= 2) {  // (more query tiles: shape 0 only)
    return launch_stream_shape<T, NT, kShapes[0].warps, kShapes[0].stages, kShapes[0].pair, kShapes[0].ctas>(km, vm, a, grid, stream);
  } else {
    switch (shape) {
#define WT_SHAPE_CASE(i)                                                                                      \
  case i:                                                                                                    \
    return launch_stream_shape<T, NT, kShapes[i].warps, kShapes[i].stages, kShapes[i].pair, kShapes[i].ctas>(km, vm, a, grid, \
                                                                                             stream);
      WT_SHAPE_CASE(0)
      WT_SHAPE_CASE(1)
      WT_SHAPE_CASE(3)
      WT_SHAPE_CASE(4)
      WT_SHAPE_CASE(5)
#undef WT_SHAPE_CASE
      default:
        return launch_stream_shape<T, NT, kShapes[2].warps, kShapes[2].stages, kShapes[2].pair, kShapes[2].ctas>(km, vm, a, grid,
                                                                                               stream);
    }
  }
}

}  // namespace

size_t cross_stream_workspace(int W, int S, int H, int Tn, int P) {
  if (P == 0 && window_kernel_ok(W, S, H, Tn)) return 256;  // (the device error word only)
  return plan_stream(W, S, H, Tn, P).bytes;
}

bool cross_stream_slices_ok(int Tn, int P) {
  // every 16-key block of every slice holds at least one key (the block math needs one)
  if (P <= 0) return false;
  const int chunk = (Tn + P - 1) / P, bpu = (chunk + 15) / 16;
  return Tn - (P - 1) * chunk > 16 * (bpu - 1);
}

int cross_stream(int dtype, const void *q, const void *k, const void *v, void *y, int W, int S, int H, int Tn,
                 void *workspace, size_t workspace_bytes, void *stream, int P, float *slices_out) {
  if (P == 0 && window_kernel_ok(W, S, H, Tn)) {
    WT_REQUIRE(static_cast<long long>(W) * H * Tn < (1LL << 31), WT_ERR_ARG, "cross_attn: too large");
    WT_REQUIRE(workspace && workspace_bytes >= 256, WT_ERR_WORKSPACE,
               "cross_attn: needs a zeroed workspace of 256 bytes (given %zu)", workspace ? workspace_bytes : 0);
    CUtensorMap km, vm;
    const unsigned long long rows = static_cast<unsigned long long>(W) * H * Tn;
    int st = encode_rows128_map(&km, k, rows, 16, dtype);
    if (st != WT_OK) return st;
    st = encode_rows128_map(&vm, v, rows, 16, dtype);
    if (st != WT_OK) return st;
    const float scale = static_cast<float>(1.0 / 8.0 * 1.4426950408889634);
    int *err = static_cast<int *>(workspace);
    if (dtype == WT_BF16) return launch_window<__nv_bfloat16>(km, vm, q, y, err, W, S, H, Tn, scale, stream);
    return launch_window<__half>(km, vm, q, y, err, W, S, H, Tn, scale, stream);
  }
  const StreamPlan p = plan_stream(W, S, H, Tn, P);
  WT_REQUIRE(workspace && workspace_bytes >= p.bytes, WT_ERR_WORKSPACE,
             "cross_attn: needs a zeroed workspace of %zu bytes (given %zu)", p.bytes, workspace ? workspace_bytes : 0);
  WT_REQUIRE(p.total < (1LL << 40), WT_ERR_ARG, "cross_attn: too large");
  CUtensorMap km, vm;
  const unsigned long long rows = static_cast<unsigned long long>(W) * H * Tn;
  int st = encode_rows128_map(&km, k, rows, 16, dtype);
  if (st != WT_OK) return st;
  st = encode_rows128_map(&vm, v, rows, 16, dtype);
  if (st != WT_OK) return st;
  char *ws = static_cast<char *>(workspace);
  StreamArgs a{q,       y,    reinterpret_cast<float *>(ws + p.part_off), reinterpret_cast<int *>(ws + p.counters_off),
               reinterpret_cast<int *>(ws), P > 0 ? slices_out : nullptr, p.slices, p.chunk, W, S, H, Tn, p.qgs,
               p.bpu, p.total, p.per_warp, p.max_slots,
               static_cast<float>(1.0 / 8.0 * 1.4426950408889634), wait_limit(), test_withhold_stage()};
  const bool bf = dtype == WT_BF16;
  const int g = p.grid, sh = p.shape;
  switch (p.nt) {
    case 1: return bf ? launch_stream_nt<__nv_bfloat16, 1>(km, vm, a, g, sh, stream) : launch_stream_nt<__half, 1>(km, vm, a, g, sh, stream);
    case 2: return bf ? launch_stream_nt<__nv_bfloat16, 2>(km, vm, a, g, sh, stream) : launch_stream_nt<__half, 2>(km, vm, a, g, sh, stream);
    case 3: return bf ? launch_stream_nt<__nv_bfloat16, 3>(km, vm, a, g, sh, stream) : launch_stream_nt<__half, 3>(km, vm, a, g, sh, stream);
    default: return bf ? launch_stream_nt<__nv_bfloat16, 4>(km, vm, a, g, sh, stream) : launch_stream_nt<__half, 4>(km, vm, a, g, sh, stream);
  }
}

}  // namespace wt
