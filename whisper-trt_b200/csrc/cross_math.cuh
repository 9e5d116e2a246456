// The tensor-core math of one 16-key block of cross-attention, shared by the cross-attention kernels:
// S^T = K Q^T (keys as M, queries as N), online softmax in log2 units, O^T += V^T P^T -- see cross_attn.cu.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace wt {

constexpr int kD = 64;

template <typename T> struct Mma;
template <> struct Mma<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// The operands of one 16-key block for one lane (g = lane / 4, c = lane % 4):
//   ka/kb: key rows g and g+8, head-dim pieces [8c, 8c+8) and [32+8c, 32+8c+8)
//   v0..v3: value rows 2c, 2c+1, 2c+8, 2c+9, head-dim piece [8g, 8g+8)
struct Block {
  uint4 ka0, kb0, ka1, kb1, v0, v1, v2, v3;
};

template <typename T>
__device__ __forceinline__ void load_block(Block &b, const T *kb, const T *vb, int k0, int hi, int g, int c) {
  const int last = hi - 1;
  const int r0 = min(k0 + g, last), r8 = min(k0 + g + 8, last);
  b.ka0 = ldg_stream(kb + static_cast<size_t>(r0) * kD + 8 * c);
  b.kb0 = ldg_stream(kb + static_cast<size_t>(r0) * kD + 32 + 8 * c);
  b.ka1 = ldg_stream(kb + static_cast<size_t>(r8) * kD + 8 * c);
  b.kb1 = ldg_stream(kb + static_cast<size_t>(r8) * kD + 32 + 8 * c);
  b.v0 = ldg_stream(vb + static_cast<size_t>(min(k0 + 2 * c, last)) * kD + 8 * g);
  b.v1 = ldg_stream(vb + static_cast<size_t>(min(k0 + 2 * c + 1, last)) * kD + 8 * g);
  b.v2 = ldg_stream(vb + static_cast<size_t>(min(k0 + 2 * c + 8, last)) * kD + 8 * g);
  b.v3 = ldg_stream(vb + static_cast<size_t>(min(k0 + 2 * c + 9, last)) * kD + 8 * g);
}

template <int NT>
struct State {
  float m[NT][2], l[NT][2], o[NT][4][4];
};

// exp2 on the special-function unit (PTX ex2.approx.ftz.f32: relative error ~2^-22, ex2(-inf) = +0).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// One 16-key block into the online-softmax state of NT tiles of 8 queries, from prepared tensor-core operands:
//   ka[s]  : A fragment (16 keys x 16 head dims) of k-step s of S^T = K Q^T
//   va[i]  : A fragment (16 head dims x 16 keys) of head-dim tile i of O^T = V^T P^T
//   qf[nt] : B fragments of the queries, k-step s in qf[nt][2s], qf[nt][2s+1]
//   ok0/ok8: keys g and g+8 of the block exist (masked to -inf otherwise)
// P enters the P.V product as hi + lo parts in the input type (two products: fp16 keeps ~22 bits of each weight,
// bf16 ~16) and the row sums use the same split values, so numerator and denominator see the same weights.
template <typename T, int NT>
__device__ __forceinline__ void attend_block(State<NT> &st, const uint32_t (&ka)[4][4], const uint32_t (&va)[4][4],
                                             const uint32_t (&qf)[NT][8], bool ok0, bool ok8, float scale) {
  constexpr bool kSplitP = true;  // P = hi + lo in the input type: ~22 bits of each weight reach the P.V product
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; ++s) Mma<T>::run(sc, ka[s][0], ka[s][1], ka[s][2], ka[s][3], qf[nt][2 * s], qf[nt][2 * s + 1]);
    // sc: (key g, query 2c), (key g, query 2c+1), (key g+8, query 2c), (key g+8, query 2c+1)
    const float s0 = ok0 ? sc[0] * scale : kNegInf, s1 = ok0 ? sc[1] * scale : kNegInf;
    const float s2 = ok8 ? sc[2] * scale : kNegInf, s3 = ok8 ? sc[3] * scale : kNegInf;
    float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(st.m[nt][0], mx0), mn1 = fmaxf(st.m[nt][1], mx1);  // finite: the block has a key
    const float a0 = ex2(st.m[nt][0] - mn0), a1 = ex2(st.m[nt][1] - mn1);
    st.m[nt][0] = mn0;
    st.m[nt][1] = mn1;
    const float p0 = ex2(s0 - mn0), p1 = ex2(s1 - mn1), p2 = ex2(s2 - mn0), p3 = ex2(s3 - mn1);
    const uint32_t h01 = Elem<T>::from_float2(p0, p1), h23 = Elem<T>::from_float2(p2, p3);
    const float2 r01 = Elem<T>::to_float2(h01), r23 = Elem<T>::to_float2(h23);
    float l0 = r01.x + r23.x, l1 = r01.y + r23.y;
    uint32_t lo01 = 0, lo23 = 0;
    if (kSplitP) {
      lo01 = Elem<T>::from_float2(p0 - r01.x, p1 - r01.y);
      lo23 = Elem<T>::from_float2(p2 - r23.x, p3 - r23.y);
      const float2 q01 = Elem<T>::to_float2(lo01), q23 = Elem<T>::to_float2(lo23);
      l0 += q01.x + q23.x;
      l1 += q01.y + q23.y;
    }
    st.l[nt][0] = st.l[nt][0] * a0 + l0;
    st.l[nt][1] = st.l[nt][1] * a1 + l1;
    const uint32_t pb0 = movmatrix_trans(h01), pb1 = movmatrix_trans(h23);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      st.o[nt][i][0] *= a0;
      st.o[nt][i][1] *= a1;
      st.o[nt][i][2] *= a0;
      st.o[nt][i][3] *= a1;
      Mma<T>::run(st.o[nt][i], va[i][0], va[i][1], va[i][2], va[i][3], pb0, pb1);
    }
    if (kSplitP) {
      const uint32_t qb0 = movmatrix_trans(lo01), qb1 = movmatrix_trans(lo23);
#pragma unroll
      for (int i = 0; i < 4; ++i) Mma<T>::run(st.o[nt][i], va[i][0], va[i][1], va[i][2], va[i][3], qb0, qb1);
    }
  }
}

// Two 16-key blocks (32 keys) into the online-softmax state at once: the two S^T products are independent mma
// chains, and the max / exp / rescale of the online softmax run once per 32 keys. ok[b][0/1]: keys g / g+8 of
// block b exist.
template <typename T, int NT>
__device__ __forceinline__ void attend_block2(State<NT> &st, const uint32_t (&ka0)[4][4], const uint32_t (&va0)[4][4],
                                              const uint32_t (&ka1)[4][4], const uint32_t (&va1)[4][4],
                                              const uint32_t (&qf)[NT][8], const bool (&ok)[2][2], float scale) {
  constexpr bool kSplitP = true;  // P = hi + lo in the input type: ~22 bits of each weight reach the P.V product
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      Mma<T>::run(c0, ka0[s][0], ka0[s][1], ka0[s][2], ka0[s][3], qf[nt][2 * s], qf[nt][2 * s + 1]);
      Mma<T>::run(c1, ka1[s][0], ka1[s][1], ka1[s][2], ka1[s][3], qf[nt][2 * s], qf[nt][2 * s + 1]);
    }
    float sv[2][4];
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const float *cc = b ? c1 : c0;
      sv[b][0] = ok[b][0] ? cc[0] * scale : kNegInf;
      sv[b][1] = ok[b][0] ? cc[1] * scale : kNegInf;
      sv[b][2] = ok[b][1] ? cc[2] * scale : kNegInf;
      sv[b][3] = ok[b][1] ? cc[3] * scale : kNegInf;
    }
    float mx0 = fmaxf(fmaxf(sv[0][0], sv[0][2]), fmaxf(sv[1][0], sv[1][2]));
    float mx1 = fmaxf(fmaxf(sv[0][1], sv[0][3]), fmaxf(sv[1][1], sv[1][3]));
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(st.m[nt][0], mx0), mn1 = fmaxf(st.m[nt][1], mx1);  // finite: block 0 has a key
    const float a0 = ex2(st.m[nt][0] - mn0), a1 = ex2(st.m[nt][1] - mn1);
    st.m[nt][0] = mn0;
    st.m[nt][1] = mn1;
    uint32_t hi[2][2], lo[2][2] = {{0u, 0u}, {0u, 0u}};
    float l0 = 0.f, l1 = 0.f;
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      const float p0 = ex2(sv[b][0] - mn0), p1 = ex2(sv[b][1] - mn1), p2 = ex2(sv[b][2] - mn0),
                  p3 = ex2(sv[b][3] - mn1);
      hi[b][0] = Elem<T>::from_float2(p0, p1);
      hi[b][1] = Elem<T>::from_float2(p2, p3);
      const float2 r01 = Elem<T>::to_float2(hi[b][0]), r23 = Elem<T>::to_float2(hi[b][1]);
      l0 += r01.x + r23.x;
      l1 += r01.y + r23.y;
      if (kSplitP) {
        lo[b][0] = Elem<T>::from_float2(p0 - r01.x, p1 - r01.y);
        lo[b][1] = Elem<T>::from_float2(p2 - r23.x, p3 - r23.y);
        const float2 q01 = Elem<T>::to_float2(lo[b][0]), q23 = Elem<T>::to_float2(lo[b][1]);
        l0 += q01.x + q23.x;
        l1 += q01.y + q23.y;
      }
    }
    st.l[nt][0] = st.l[nt][0] * a0 + l0;
    st.l[nt][1] = st.l[nt][1] * a1 + l1;
    const uint32_t p00 = movmatrix_trans(hi[0][0]), p01 = movmatrix_trans(hi[0][1]);
    const uint32_t p10 = movmatrix_trans(hi[1][0]), p11 = movmatrix_trans(hi[1][1]);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      st.o[nt][i][0] *= a0;
      st.o[nt][i][1] *= a1;
      st.o[nt][i][2] *= a0;
      st.o[nt][i][3] *= a1;
      Mma<T>::run(st.o[nt][i], va0[i][0], va0[i][1], va0[i][2], va0[i][3], p00, p01);
      Mma<T>::run(st.o[nt][i], va1[i][0], va1[i][1], va1[i][2], va1[i][3], p10, p11);
    }
    if (kSplitP) {
      const uint32_t q00 = movmatrix_trans(lo[0][0]), q01 = movmatrix_trans(lo[0][1]);
      const uint32_t q10 = movmatrix_trans(lo[1][0]), q11 = movmatrix_trans(lo[1][1]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        Mma<T>::run(st.o[nt][i], va0[i][0], va0[i][1], va0[i][2], va0[i][3], q00, q01);
        Mma<T>::run(st.o[nt][i], va1[i][0], va1[i][1], va1[i][2], va1[i][3], q10, q11);
      }
    }
  }
}

// --- operands loaded straight from HBM (register-direct; head dims permuted) ----------------------------------
// Key fragments: lane (g, c) holds key rows g, g+8, head dims [8c, 8c+8) and [32+8c, 32+8c+8); k-step s uses
// words (s%2)*2, (s%2)*2+1 of the first (s < 2) or second piece -- the queries use the same permutation.
// Value fragments: value rows 2c, 2c+1, 2c+8, 2c+9, head dims [8g, 8g+8), paired by byte permutes; head-dim tile
// i, row g / g+8 of the O^T accumulator is head dim 8g+2i / 8g+2i+1.
template <typename T, int NT>
__device__ __forceinline__ void compute_block(State<NT> &st, const Block &b, const uint32_t (&qf)[NT][8], int k0,
                                              int hi, int g, float scale) {
  uint32_t ka[4][4], va[4][4];
  ka[0][0] = b.ka0.x; ka[0][1] = b.ka1.x; ka[0][2] = b.ka0.y; ka[0][3] = b.ka1.y;
  ka[1][0] = b.ka0.z; ka[1][1] = b.ka1.z; ka[1][2] = b.ka0.w; ka[1][3] = b.ka1.w;
  ka[2][0] = b.kb0.x; ka[2][1] = b.kb1.x; ka[2][2] = b.kb0.y; ka[2][3] = b.kb1.y;
  ka[3][0] = b.kb0.z; ka[3][1] = b.kb1.z; ka[3][2] = b.kb0.w; ka[3][3] = b.kb1.w;
  const uint32_t w0[4] = {b.v0.x, b.v0.y, b.v0.z, b.v0.w}, w1[4] = {b.v1.x, b.v1.y, b.v1.z, b.v1.w};
  const uint32_t w2[4] = {b.v2.x, b.v2.y, b.v2.z, b.v2.w}, w3[4] = {b.v3.x, b.v3.y, b.v3.z, b.v3.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    va[i][0] = __byte_perm(w0[i], w1[i], 0x5410);
    va[i][1] = __byte_perm(w0[i], w1[i], 0x7632);
    va[i][2] = __byte_perm(w2[i], w3[i], 0x5410);
    va[i][3] = __byte_perm(w2[i], w3[i], 0x7632);
  }
  attend_block<T, NT>(st, ka, va, qf, (k0 + g) < hi, (k0 + g + 8) < hi, scale);
}

// --- operands from shared memory (TMA tiles, 128-byte swizzle; standard fragment layout) ------------------------
// A 16-row tile of 128-byte rows written by a 2D TMA load with 128-byte swizzle holds chunk c of row r at chunk
// c ^ (r % 8). ldmatrix reads it without bank conflicts (each 8x8 matrix = 8 rows of one chunk = 8 distinct chunk
// positions). Key fragments with ldmatrix.x4, value fragments transposed with ldmatrix.x4.trans; head dims in
// natural order (head-dim tile i, accumulator row g / g+8 = head dim 16i+g / 16i+g+8).
__device__ __forceinline__ int swizzle128(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const unsigned char *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const unsigned char *p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(static_cast<uint32_t>(__cvta_generic_to_shared(p))));
}

__device__ __forceinline__ void smem_frags(uint32_t (&ka)[4][4], uint32_t (&va)[4][4], const unsigned char *kt,
                                           const unsigned char *vt, int lane) {
  const int r8 = lane & 7, m = lane >> 3;
  // K (A of S^T = K Q^T): matrices (rows 0-7, dims lo), (rows 8-15, lo), (rows 0-7, hi), (rows 8-15, hi)
  const int krow = r8 + ((m & 1) << 3), kchunk_hi = m >> 1;
#pragma unroll
  for (int s = 0; s < 4; ++s) ldmatrix_x4(ka[s], kt + swizzle128(krow, 2 * s + kchunk_hi));
  // V^T (A of O^T = V^T P^T), transposed: matrices (keys 0-7, dims lo), (keys 0-7, hi), (keys 8-15, lo), (8-15, hi)
  const int vrow = r8 + ((m >> 1) << 3), vchunk_hi = m & 1;
#pragma unroll
  for (int i = 0; i < 4; ++i) ldmatrix_x4_trans(va[i], vt + swizzle128(vrow, 2 * i + vchunk_hi));
}

// Query B fragments in the standard layout: lane (g, c) holds query g's head-dim pairs (16s+2c, +1) and
// (16s+2c+8, +9), i.e. 32-bit words c + 4j (j = 0..7) of the query row.
template <typename T, int NT>
__device__ __forceinline__ void load_q_std(uint32_t (&qf)[NT][8], const T *qrow0, size_t qstride, int q0, int S,
                                           int g, int c) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int qi = q0 + nt * 8 + g;
    if (qi < S) {
      const uint32_t *w = reinterpret_cast<const uint32_t *>(qrow0 + static_cast<size_t>(qi) * qstride);
#pragma unroll
      for (int j = 0; j < 8; ++j) qf[nt][j] = __ldg(w + c + 4 * j);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) qf[nt][j] = 0u;
    }
  }
}

}  // namespace wt
