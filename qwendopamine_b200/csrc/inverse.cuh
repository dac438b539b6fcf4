// inverse.cuh -- unit-lower triangular inverse of a 64 x 64 chunk matrix.
#pragma once

#include "common.cuh"

namespace gdn2 {

// Unit-lower inverse of (I + L) for a 64x64 strictly-lower L held in sL
// (row stride LDC); the result goes to sInv.  sTmp holds 3 16x16 blocks.
// Diagonal 16x16 blocks by forward substitution (one warp each), then the
// off-diagonal blocks level by level:  Inv_IJ = -Inv_II sum_{J<=M<I} L_IM Inv_MJ.
template <int LDC>
__device__ void unit_lower_inverse(const float* sL, float* sInv, float* sTmp) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int idx = tid; idx < kChunk * LDC; idx += blockDim.x) sInv[idx] = 0.f;
  __syncthreads();
  if (warp < 4 && lane < 16) {
    const int o = warp * 16, j = lane;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float s = (r == j) ? 1.f : 0.f;
#pragma unroll
      for (int i = 0; i < r; ++i) s -= sL[(o + r) * LDC + o + i] * x[i];
      x[r] = s;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) sInv[(o + r) * LDC + o + j] = x[r];
  }
  __syncthreads();
  for (int d = 1; d < 4; ++d) {
    const int nb = 4 - d;  // blocks (I, J=I-d) for I = d..3
    // T_b = sum_{x=16J}^{16I-1} L[16I+r][x] * Inv[x][16J+c]
    for (int idx = tid; idx < nb * 256; idx += blockDim.x) {
      int bI = d + idx / 256, bJ = bI - d, e = idx & 255, r = e >> 4, c = e & 15;
      float s = 0.f;
      for (int x = 16 * bJ; x < 16 * bI; ++x) s += sL[(16 * bI + r) * LDC + x] * sInv[x * LDC + 16 * bJ + c];
      sTmp[idx] = s;
    }
    __syncthreads();
    for (int idx = tid; idx < nb * 256; idx += blockDim.x) {
      int bI = d + idx / 256, bJ = bI - d, e = idx & 255, r = e >> 4, c = e & 15;
      const float* t = sTmp + (idx / 256) * 256;
      float s = 0.f;
#pragma unroll
      for (int m = 0; m < 16; ++m) s += sInv[(16 * bI + r) * LDC + 16 * bI + m] * t[m * 16 + c];
      sInv[(16 * bI + r) * LDC + 16 * bJ + c] = -s;
    }
    __syncthreads();
  }
}

// acc (16 x 16) = A (16 x KD) B (KD x 16) on the tensor cores, TERMS = 3:
// the 3-term TF32 split (hi*hi + hi*lo + lo*hi, about fp32 accuracy; the
// three accumulator chains run independently); TERMS = 1: plain TF32
// operands, fp32 accumulation (the precision the reference's solve_tril
// products use on GPUs of this class, chunk_gdn2.py:464).
// A(m,k) = A[m*lda + k], B(k,n) = B[k*ldb + n] (fp32 shared memory).
template <int KD, int TERMS = 3>
__device__ __forceinline__ void mma16x16_tf32x3(float (&acc)[1][2][4], const float* A, int lda,
                                                const float* B, int ldb) {
  static_assert(TERMS == 1 || TERMS == 3, "TF32 terms");
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  float hh[2][4], lh[2][4], hl[2][4];
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) hh[j][e] = lh[j][e] = hl[j][e] = 0.f;
#pragma unroll
  for (int k0 = 0; k0 < KD; k0 += 8) {
    const float* a = A + gid * lda + k0 + tig;
    const float x[4] = {a[0], a[8 * lda], a[4], a[8 * lda + 4]};
    uint32_t ah[4], al[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      ah[e] = tf32_bits(x[e]);
      al[e] = tf32_bits(x[e] - __uint_as_float(ah[e]));
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float* bp = B + (k0 + tig) * ldb + j * 8 + gid;
      const float y0 = bp[0], y1 = bp[4 * ldb];
      const uint32_t bh0 = tf32_bits(y0), bh1 = tf32_bits(y1);
      const uint32_t bl0 = tf32_bits(y0 - __uint_as_float(bh0));
      const uint32_t bl1 = tf32_bits(y1 - __uint_as_float(bh1));
      mma_tf32(hh[j], ah, bh0, bh1);
      if (TERMS == 3) {
        mma_tf32(lh[j], al, bh0, bh1);
        mma_tf32(hl[j], ah, bl0, bl1);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[0][j][e] = hh[j][e] + (lh[j][e] + hl[j][e]);
}

// Blocks at distance d = I - J of the inverse, one warp per block:
//   T = sum_{M=J}^{I-1} L_IM Inv_MJ,   Inv_IJ = -Inv_II T.
template <int LDC, int DIST, int TERMS>
__device__ __forceinline__ void inverse_level(const float* sL, float* sInv, float* sT) {
  const int warp = threadIdx.x >> 5;
  if (warp < 4 - DIST) {
    const int J = warp, I = warp + DIST;
    float* t = sT + warp * (16 * 20);
    float acc[1][2][4];
    mma16x16_tf32x3<16 * DIST, TERMS>(acc, sL + 16 * I * LDC + 16 * J, LDC,
                                      sInv + 16 * J * LDC + 16 * J, LDC);
    acc_foreach(acc, [&](int r, int c, float v) { t[r * 20 + c] = v; });
    __syncwarp();
    mma16x16_tf32x3<16, TERMS>(acc, sInv + 16 * I * LDC + 16 * I, LDC, t, 20);
    acc_foreach(acc, [&](int r, int c, float v) { sInv[(16 * I + r) * LDC + 16 * J + c] = -v; });
  }
}

// Same inverse for CTAs of >= 4 warps, reading only the strictly-lower
// blocks of sL (the upper blocks of sL and of sInv are neither read nor
// written; callers treat them as zero).  The diagonal 16x16 blocks are
// solved right-looking in registers (lane j of warp I holds column j of
// Inv_II, so the dependent chain is one FMA per row); the off-diagonal blocks
// follow by distance with TF32 tensor-core products (inverse_level; TERMS as
// for mma16x16_tf32x3).  sT holds 3 [16][20] fp32 tiles.
template <int LDC, int TERMS = 3>
__device__ void unit_lower_inverse_mma(const float* sL, float* sInv, float* sT) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < 4 && lane < 16) {
    const int o = 16 * warp, j = lane;
    const float* Lb = sL + o * LDC + o;
    float x[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) x[r] = (r == j) ? 1.f : 0.f;
#pragma unroll
    for (int i = 0; i < 15; ++i)
#pragma unroll
      for (int r = i + 1; r < 16; ++r) x[r] -= Lb[r * LDC + i] * x[i];
#pragma unroll
    for (int r = 0; r < 16; ++r) sInv[(o + r) * LDC + o + j] = x[r];
  }
  __syncthreads();
  inverse_level<LDC, 1, TERMS>(sL, sInv, sT);
  __syncthreads();
  inverse_level<LDC, 2, TERMS>(sL, sInv, sT);
  __syncthreads();
  inverse_level<LDC, 3, TERMS>(sL, sInv, sT);
  __syncthreads();
}

}  // namespace gdn2
