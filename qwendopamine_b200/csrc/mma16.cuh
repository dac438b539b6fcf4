// mma16.cuh -- 16-bit tensor-core tiles from shared memory (bf16 / fp16).
//
// Operands live in shared memory as row-major 16-bit tiles whose row pitch is
// a multiple of 16 bytes and not a multiple of 128 bytes (e.g. D + 8
// elements), so ldmatrix row fetches are bank-conflict free.  A warp computes
// acc[(16*MT) x (8*NT)] (fp32) += A[(16*MT) x kd] * B[kd x (8*NT)] with
// mma.sync m16n8k16 and fp32 accumulation; ldmatrix (.trans when needed)
// turns either storage orientation of A or B into the register fragments:
//   A_KMAJOR:  A(m,k) = A[m*lda + k]   (else A(m,k) = A[k*lda + m])
//   B_KMAJOR:  B(k,n) = B[n*ldb + k]   (else B(k,n) = B[k*ldb + n])
// Also: cp.async 16-byte global->shared copies with zero fill.
#pragma once

#include "common.cuh"

namespace gdn2 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];\n"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(smem_u32(p)));
}

template <typename T> struct Mma16;
template <> struct Mma16<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <> struct Mma16<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

// A fragment (16 x 16 at rows m0, cols k0 of the logical A).
template <bool A_KMAJOR, typename T>
__device__ __forceinline__ void load_a16(uint32_t (&a)[4], const T* A, int lda, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  if (A_KMAJOR) {
    const int r = m0 + (lane & 15), c = k0 + ((lane >> 4) << 3);
    ldsm_x4(a, A + r * lda + c);
  } else {
    const int j = lane >> 3, rr = lane & 7;
    const int k = k0 + rr + ((j >> 1) << 3), m = m0 + ((j & 1) << 3);
    ldsm_x4_t(a, A + k * lda + m);
  }
}

// Two B fragments (k0..k0+15 x n0..n0+15): b[0],b[1] for n0..n0+7 and
// b[2],b[3] for n0+8..n0+15.
template <bool B_KMAJOR, typename T>
__device__ __forceinline__ void load_b16x2(uint32_t (&b)[4], const T* B, int ldb, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  const int j = lane >> 3, rr = lane & 7;
  if (B_KMAJOR) {
    const int n = n0 + rr + ((j >> 1) << 3), k = k0 + ((j & 1) << 3);
    ldsm_x4(b, B + n * ldb + k);
  } else {
    const int k = k0 + rr + ((j & 1) << 3), n = n0 + ((j >> 1) << 3);
    ldsm_x4_t(b, B + k * ldb + n);
  }
}

// acc[16*MT x 8*NT] += A[rows m0.., k 0..kd) * B[k 0..kd, cols n0..); NT even.
template <int MT, int NT, bool A_KMAJOR, bool B_KMAJOR, typename T>
__device__ __forceinline__ void warp_mma16(float (&acc)[MT][NT][4], const T* A, int lda, int m0,
                                           const T* B, int ldb, int n0, int kd) {
  static_assert(NT % 2 == 0, "NT must be even");
#pragma unroll
  for (int k0 = 0; k0 < kd; k0 += 16) {
    uint32_t a[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) load_a16<A_KMAJOR>(a[i], A, lda, m0 + 16 * i, k0);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      load_b16x2<B_KMAJOR>(b, B, ldb, k0, n0 + 8 * j);
#pragma unroll
      for (int i = 0; i < MT; ++i) {
        Mma16<T>::run(acc[i][j], a[i], b[0], b[1]);
        Mma16<T>::run(acc[i][j + 1], a[i], b[2], b[3]);
      }
    }
  }
}

// acc (16 x 8) += A[rows m0.., k 0..kd) * B[k 0..kd, cols n0..n0+7) with B
// K-major (row n holds B[., n]): one n8 tile per warp.
template <bool A_KMAJOR, typename T>
__device__ __forceinline__ void warp_mma16_n8(float (&acc)[4], const T* A, int lda, int m0,
                                              const T* B, int ldb, int n0, int kd) {
  const int lane = threadIdx.x & 31;
  const int rr = lane & 7, kh = (lane >> 3) & 1;
#pragma unroll
  for (int k0 = 0; k0 < kd; k0 += 16) {
    uint32_t a[4], b[2];
    load_a16<A_KMAJOR>(a, A, lda, m0, k0);
    ldsm_x2(b, B + (n0 + rr) * ldb + k0 + 8 * kh);
    Mma16<T>::run(acc, a, b[0], b[1]);
  }
}

// acc1 += A1 B and acc2 += A2 B with the B fragments loaded once (the two A
// tiles share lda / m0 / kd).
template <int NT, bool A_KMAJOR, bool B_KMAJOR, typename T>
__device__ __forceinline__ void warp_mma16_2a(float (&acc1)[1][NT][4], float (&acc2)[1][NT][4],
                                              const T* A1, const T* A2, int lda, int m0,
                                              const T* B, int ldb, int n0, int kd) {
  static_assert(NT % 2 == 0, "NT must be even");
#pragma unroll
  for (int k0 = 0; k0 < kd; k0 += 16) {
    uint32_t a1[4], a2[4];
    load_a16<A_KMAJOR>(a1, A1, lda, m0, k0);
    load_a16<A_KMAJOR>(a2, A2, lda, m0, k0);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      load_b16x2<B_KMAJOR>(b, B, ldb, k0, n0 + 8 * j);
      Mma16<T>::run(acc1[0][j], a1, b[0], b[1]);
      Mma16<T>::run(acc1[0][j + 1], a1, b[2], b[3]);
      Mma16<T>::run(acc2[0][j], a2, b[0], b[1]);
      Mma16<T>::run(acc2[0][j + 1], a2, b[2], b[3]);
    }
  }
}

// ---- the same fragments from 128-byte-swizzled tiles ------------------------
// Tiles of 64 16-bit elements per 128-byte row as TMA writes them with
// 128-byte swizzle (the 16-byte chunk c of row r sits at chunk c ^ (r & 7));
// `col` is a multiple of 8.
__device__ __forceinline__ const void* sw128(const void* base, int row, int col) {
  return static_cast<const unsigned char*>(base) + row * 128 + ((((col >> 3) ^ (row & 7))) << 4);
}
// Element address inside such a tile (any col).
template <typename T>
__device__ __forceinline__ const T* sw128_elem(const T* base, int row, int col) {
  return reinterpret_cast<const T*>(sw128(base, row, col & ~7)) + (col & 7);
}
template <bool A_KMAJOR, typename T>
__device__ __forceinline__ void load_a16_sw(uint32_t (&a)[4], const T* A, int m0, int k0) {
  const int lane = threadIdx.x & 31;
  if (A_KMAJOR) {
    ldsm_x4(a, sw128(A, m0 + (lane & 15), k0 + ((lane >> 4) << 3)));
  } else {
    const int j = lane >> 3, rr = lane & 7;
    ldsm_x4_t(a, sw128(A, k0 + rr + ((j >> 1) << 3), m0 + ((j & 1) << 3)));
  }
}
template <bool B_KMAJOR, typename T>
__device__ __forceinline__ void load_b16x2_sw(uint32_t (&b)[4], const T* B, int k0, int n0) {
  const int lane = threadIdx.x & 31;
  const int j = lane >> 3, rr = lane & 7;
  if (B_KMAJOR)
    ldsm_x4(b, sw128(B, n0 + rr + ((j >> 1) << 3), k0 + ((j & 1) << 3)));
  else
    ldsm_x4_t(b, sw128(B, k0 + rr + ((j & 1) << 3), n0 + ((j >> 1) << 3)));
}

// Pack two floats into a 16-bit pair (low half = first).
template <typename T> __device__ __forceinline__ uint32_t pack2(float x, float y);
template <> __device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float x, float y) {
  __nv_bfloat162 v = __floats2bfloat162_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack2<__half>(float x, float y) {
  __half2 v = __floats2half2_rn(x, y);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Two adjacent elements (the first 4- or 8-byte aligned) as floats: one
// shared-memory access instead of two.
template <typename T> __device__ __forceinline__ float2 ld2(const T* p);
template <> __device__ __forceinline__ float2 ld2<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
}
template <> __device__ __forceinline__ float2 ld2<__half>(const __half* p) {
  return __half22float2(*reinterpret_cast<const __half2*>(p));
}
template <> __device__ __forceinline__ float2 ld2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
// The two 16-bit elements of a 32-bit word as floats.
template <typename T> __device__ __forceinline__ float2 unpack2(uint32_t x) {
  return ld2<T>(reinterpret_cast<const T*>(&x));
}

// Packed fp32x2 arithmetic: one instruction for both elements of a column
// pair, each rounded as the scalar operation is.  pr / setpr view elements
// (2 hf, 2 hf + 1) of an mma fragment -- one row, two adjacent columns -- as
// such a pair.
__device__ __forceinline__ float2 f2(float s) { return make_float2(s, s); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }
__device__ __forceinline__ float2 exp2_2(float2 x) {
  return make_float2(fast_exp2(x.x), fast_exp2(x.y));
}
__device__ __forceinline__ float2 pr(const float (&a)[4], int hf) {
  return make_float2(a[2 * hf], a[2 * hf + 1]);
}
__device__ __forceinline__ void setpr(float (&a)[4], int hf, float2 v) {
  a[2 * hf] = v.x;
  a[2 * hf + 1] = v.y;
}

// ---------------------------------------------------------------------------
// cp.async
// ---------------------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Copy a ROWS x COLS 16-bit tile (global row stride ldg elements, 16-byte
// aligned rows) into shared memory (row stride lds), asynchronously.  Rows
// >= nrows / cols >= ncols (ncols a multiple of 8) are zero-filled.
template <typename T, int ROWS, int COLS, int NTH>
__device__ __forceinline__ void cp_tile16(T* s, int lds, const T* g, int64_t ldg, int nrows,
                                          int ncols) {
  constexpr int CPR = COLS / 8;
  constexpr int TOTAL = ROWS * CPR;
#pragma unroll
  for (int it = 0; it < (TOTAL + NTH - 1) / NTH; ++it) {
    const int idx = threadIdx.x + it * NTH;
    if (idx < TOTAL) {
      const int r = idx / CPR, c = (idx - r * CPR) * 8;
      const bool ok = r < nrows && c < ncols;
      cp_async16(s + r * lds + c, ok ? (const void*)(g + (int64_t)r * ldg + c) : (const void*)g,
                 ok);
    }
  }
}

// Segmented inclusive scan down the 64 rows of an fp32 tile with NC columns
// (row stride lds) using NTH threads: prefix sums (REV false) or suffix sums
// (REV true), times mul.  Thread (column, segment) loads its segment of rows,
// scans it in registers, adds the totals of the earlier segments (from
// `tmp`, NTH floats) and writes each element once.  Contains __syncthreads().
template <int NC, int NTH, bool REV>
__device__ __forceinline__ void col_scan64_reg(float* s, int lds, float* tmp, float mul) {
  constexpr int NSEG = NTH / NC;
  constexpr int RPS = kChunk / NSEG;
  static_assert(NSEG * NC == NTH && RPS * NSEG == kChunk, "scan shape");
  const int col = threadIdx.x % NC, seg = threadIdx.x / NC;
  float x[RPS];
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    const int r = REV ? (kChunk - 1 - (seg * RPS + i)) : (seg * RPS + i);
    x[i] = s[r * lds + col];
  }
#pragma unroll
  for (int i = 1; i < RPS; ++i) x[i] += x[i - 1];
  tmp[seg * NC + col] = x[RPS - 1];
  __syncthreads();
  float off = 0.f;
#pragma unroll
  for (int j = 0; j < NSEG - 1; ++j)
    if (j < seg) off += tmp[j * NC + col];
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    const int r = REV ? (kChunk - 1 - (seg * RPS + i)) : (seg * RPS + i);
    s[r * lds + col] = (x[i] + off) * mul;
  }
  __syncthreads();
}

// Sums over the warp's 32 lanes of eight values per lane, reduce-scatter
// order (4 + 2 + 1 + 1 + 1 = 9 shuffles instead of 8 x 5): returns the total
// of value idx = 4 * bit4 + 2 * bit3 + bit2 of the lane id, held by the 4
// lanes that share those bits.
__device__ __forceinline__ float warp_reduce8(const float (&v)[8], int lane) {
  const bool h4 = lane & 16, h3 = lane & 8, h2 = lane & 4;
  float a[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = h4 ? v[i] : v[4 + i];
    a[i] = (h4 ? v[4 + i] : v[i]) + __shfl_xor_sync(0xffffffffu, send, 16);
  }
  float b2[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = h3 ? a[i] : a[2 + i];
    b2[i] = (h3 ? a[2 + i] : a[i]) + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  const float send = h2 ? b2[0] : b2[1];
  float c = (h2 ? b2[1] : b2[0]) + __shfl_xor_sync(0xffffffffu, send, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
  return c;
}

// Row norms of the 64-row q and k tiles (row stride ld): each warp owns
// 64 / (NTH/32) consecutive rows and reduces them together.
// rq[r] = rsqrt(sum q^2 + eps) (1 without l2norm), same for rk.
template <typename T, int D, int NTH>
__device__ __forceinline__ void row_norms16(const T* sq, const T* sk, int ld, float* rq, float* rk,
                                            int l2norm) {
  constexpr int RPW = kChunk / (NTH / 32);
  constexpr int EPL = D / 32;
  static_assert(RPW * (NTH / 32) == kChunk && RPW <= 32 && EPL * 32 == D, "norm shape");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float s1[RPW], s2[RPW];
#pragma unroll
  for (int rr = 0; rr < RPW; ++rr) {
    const int r = RPW * warp + rr;
    s1[rr] = 0.f;
    s2[rr] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float x = to_f<T>(sq[r * ld + EPL * lane + e]);
      const float y = to_f<T>(sk[r * ld + EPL * lane + e]);
      s1[rr] += x * x;
      s2[rr] += y * y;
    }
  }
  if constexpr (RPW == 4) {
    const float v[8] = {s1[0], s1[1], s1[2], s1[3], s2[0], s2[1], s2[2], s2[3]};
    const float tot = warp_reduce8(v, lane);
    if ((lane & 3) == 0) {
      const int idx = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
      const int r = RPW * warp + (idx & 3);
      (idx < 4 ? rq : rk)[r] = l2norm ? rsqrtf(tot + kNormEps) : 1.f;
    }
  } else {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int rr = 0; rr < RPW; ++rr) {
        s1[rr] += __shfl_xor_sync(0xffffffffu, s1[rr], o);
        s2[rr] += __shfl_xor_sync(0xffffffffu, s2[rr], o);
      }
#pragma unroll
    for (int rr = 0; rr < RPW; ++rr)
      if (lane == rr) {
        const int r = RPW * warp + rr;
        rq[r] = l2norm ? rsqrtf(s1[rr] + kNormEps) : 1.f;
        rk[r] = l2norm ? rsqrtf(s2[rr] + kNormEps) : 1.f;
      }
  }
}

// Per-16-row-block decay factors F[I(I+1)/2 + J][c] = 2^(G_16I - G_(16J+15))
// for J <= I (exponent capped at 120; only the diagonal pairs can be
// positive), from the log2 cumulative decay tile G (row stride ldg).
template <int D, int NTH>
__device__ __forceinline__ void block_factors(const float* G, int ldg, float* F) {
  for (int i = threadIdx.x; i < 10 * D; i += NTH) {
    const int q = i / D, cc = i - q * D;
    const int I = q >= 6 ? 3 : q >= 3 ? 2 : q >= 1 ? 1 : 0;
    const int J = q - I * (I + 1) / 2;
    F[i] = fast_exp2(fminf(G[16 * I * ldg + cc] - G[(16 * J + 15) * ldg + cc], 120.f));
  }
}

// Scale the two 16-bit values packed in x by (f.x, f.y).
template <typename T>
__device__ __forceinline__ uint32_t scale_pair(uint32_t x, float2 f) {
  const T* v = reinterpret_cast<const T*>(&x);
  return pack2<T>(to_f<T>(v[0]) * f.x, to_f<T>(v[1]) * f.y);
}

// Copy a ROWS x COLS 16-bit tile from shared memory (row stride lds) to
// global memory (row stride ldg elements, 16-byte aligned rows): rows <
// nrows, columns < ncols (a multiple of 8).  Each thread moves 16 bytes, so a
// warp instruction writes whole rows instead of fragment-shaped pieces.
template <typename T, int ROWS, int COLS, int NTH>
__device__ __forceinline__ void store_tile16(T* g, int64_t ldg, const T* s, int lds, int nrows,
                                             int ncols) {
  constexpr int CPR = COLS / 8;
  constexpr int TOTAL = ROWS * CPR;
#pragma unroll
  for (int it = 0; it < (TOTAL + NTH - 1) / NTH; ++it) {
    const int idx = threadIdx.x + it * NTH;
    if (idx < TOTAL) {
      const int r = idx / CPR, c = (idx - r * CPR) * 8;
      if (r < nrows && c < ncols)
        *reinterpret_cast<uint4*>(g + (int64_t)r * ldg + c) =
            *reinterpret_cast<const uint4*>(s + r * lds + c);
    }
  }
}

// Same for an fp32 vector of n floats (n a multiple of 4), zero beyond n.
template <int N, int NTH>
__device__ __forceinline__ void cp_vec32(float* s, const float* g, int n) {
  constexpr int CH = N / 4;
  for (int idx = threadIdx.x; idx < CH; idx += NTH) {
    const bool ok = idx * 4 < n;
    cp_async16(s + idx * 4, ok ? (const void*)(g + idx * 4) : (const void*)g, ok);
  }
}

}  // namespace gdn2
