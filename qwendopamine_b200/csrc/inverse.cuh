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

// Same inverse for CTAs of >= 4 warps, reading only the strictly-lower
// blocks of sL (the upper blocks of sL and of sInv are neither read nor
// written; callers treat them as zero).  The diagonal 16x16 blocks are
// solved right-looking in registers (lane j of warp I holds column j of
// Inv_II, so the dependent chain is one FMA per row); the off-diagonal blocks
// follow by distance d = I - J with one warp per block and 3-pass TF32
// tensor-core products (about fp32 accuracy):
//   T = sum_{M=J}^{I-1} L_IM Inv_MJ,   Inv_IJ = -Inv_II T.
// sT holds 3 [16][20] fp32 tiles.
template <int LDC>
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
  for (int d = 1; d < 4; ++d) {
    if (warp < 4 - d) {
      const int J = warp, I = warp + d;
      float* t = sT + warp * (16 * 20);
      float acc[1][2][4];
      acc_zero(acc);
      warp_mma<1, 2, 3>(acc, sL + 16 * I * LDC + 16 * J, LDC, 1, sInv + 16 * J * LDC + 16 * J, LDC,
                        1, 16 * d);
      acc_foreach(acc, [&](int r, int c, float v) { t[r * 20 + c] = v; });
      __syncwarp();
      float acc2[1][2][4];
      acc_zero(acc2);
      warp_mma<1, 2, 3>(acc2, sInv + 16 * I * LDC + 16 * I, LDC, 1, t, 20, 1, 16);
      acc_foreach(acc2, [&](int r, int c, float v) { sInv[(16 * I + r) * LDC + 16 * J + c] = -v; });
    }
    __syncthreads();
  }
}

}  // namespace gdn2
