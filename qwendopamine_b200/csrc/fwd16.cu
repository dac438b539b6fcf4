// fwd16.cu -- intra-chunk forward solve for bf16 inputs.
//
// One CTA of 16 warps per (chunk, head); same mathematics as k_fwd_intra
// (chunk_fwd.cu).  One cp.async round trip brings q, k, b, v, w and g.  The
// score operands are 16-bit tiles scaled by relative decays:
//   Qs[r] = scale q_n[r] 2^(G_r - G_b(r)),  KBs[r] = (b k_n)[r] 2^(G_r - G_b(r))
// (b(r): first row of r's 16-row block) and, for block row I, the keys
//   Ks_I[i] = k_n[i] 2^(G_16I - G_i), i < 16(I+1),
// so that every product of an Aqk / Akk block carries exactly
// 2^(G_r - G_i).  The scores, W = A E and U = A Z are mma.sync m16n8k16
// products from ldmatrix fragments; the unit-lower inverse A = (I+Akk)^-1
// stays in fp32.  Diagonal blocks whose 16-row decay range exceeds the fp32
// exponent budget are recomputed elementwise.
#include "chunk_args.cuh"
#include "inverse.cuh"
#include "mma16.cuh"

namespace gdn2 {

constexpr int kThreadsF16 = 512;

template <int D>
struct Fwd16Layout {
  static constexpr int LDK = D + 8;
  static constexpr int LDG = D + 4;
  static constexpr int LDC = kChunk + 8;   // 16-bit 64 x 64
  static constexpr int LDF = kChunk + 4;   // fp32 64 x 64
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + kChunk * LDK * 2;
  static constexpr int oB = oK + kChunk * LDK * 2;
  static constexpr int oV = oB + kChunk * LDK * 2;
  static constexpr int oW = oV + kChunk * LDK * 2;
  static constexpr int oG = oW + kChunk * LDK * 2;
  static constexpr int oMisc = oG + kChunk * LDG * 4;
  static constexpr int nMisc = 64 + 64 + 4;
  static constexpr int oR = oMisc + nMisc * 4;  // work region
  // scores
  static constexpr int rQs = 0;
  static constexpr int rKBs = rQs + kChunk * LDK * 2;
  static constexpr int rKs = rKBs + kChunk * LDK * 2;
  static constexpr int rAkk = rKs + 160 * LDK * 2;
  static constexpr int rEndScores = rAkk + kChunk * LDF * 4;
  // inverse (Akk stays in place)
  static constexpr int rInv = 0;
  static constexpr int rTmp = rInv + kChunk * LDF * 4;
  // W, U
  static constexpr int rA16 = rTmp + 3 * 256 * 4;
  static constexpr int rE = rA16 + kChunk * LDC * 2;
  static constexpr int rZ = rE + kChunk * LDK * 2;
  static constexpr int rEndWU = rZ + kChunk * LDK * 2;
  // sA16 / sE / sZ are written only after the inverse has finished reading
  // Akk, so they may overlap it; they never overlap sInv or each other.
  static constexpr int R = rEndScores > rEndWU ? rEndScores : rEndWU;
  static constexpr size_t bytes = (size_t)oR + R;
  static_assert(oR % 16 == 0 && rAkk % 16 == 0 && rA16 % 16 == 0, "alignment");
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreadsF16, 1) k_fwd_intra16(FwdIntraArgs a) {
  using L = Fwd16Layout<D>;
  constexpr int LDK = L::LDK, LDG = L::LDG, LDC = L::LDC, LDF = L::LDF;
  constexpr int NTH = kThreadsF16;
  constexpr int DQ = D / 4, NTO = DQ / 8;
  extern __shared__ __align__(16) unsigned char sm[];
  T* sq = reinterpret_cast<T*>(sm + L::oQ);
  T* sk = reinterpret_cast<T*>(sm + L::oK);
  T* sb = reinterpret_cast<T*>(sm + L::oB);
  T* sv = reinterpret_cast<T*>(sm + L::oV);
  T* sw = reinterpret_cast<T*>(sm + L::oW);
  float* sG = reinterpret_cast<float*>(sm + L::oG);
  float* rq = reinterpret_cast<float*>(sm + L::oMisc);
  float* rk = rq + 64;
  int* sFlag = reinterpret_cast<int*>(rk + 64);
  unsigned char* R = sm + L::oR;
  T* sQs = reinterpret_cast<T*>(R + L::rQs);
  T* sKBs = reinterpret_cast<T*>(R + L::rKBs);
  T* sKs = reinterpret_cast<T*>(R + L::rKs);
  float* sAkk = reinterpret_cast<float*>(R + L::rAkk);

  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int wr = warp & 3, wc = warp >> 2;
  const int H = a.H, K = a.K, V = a.V;
  const ChunkPos cp = chunk_pos(a.seqs, c);
  const int len = cp.len;
  const int64_t ldk = (int64_t)H * K, ldv = (int64_t)H * V;
  const int64_t offk = cp.row0 * ldk + (int64_t)h * K;
  const int64_t offv = cp.row0 * ldv + (int64_t)h * V;
  const size_t ch = (size_t)c * H + h;
  const float scale = a.scale;

  // ---- loads --------------------------------------------------------------
  cp_tile16<T, kChunk, D, NTH>(sq, LDK, reinterpret_cast<const T*>(a.q) + offk, ldk, len, K);
  cp_tile16<T, kChunk, D, NTH>(sk, LDK, reinterpret_cast<const T*>(a.k) + offk, ldk, len, K);
  cp_tile16<T, kChunk, D, NTH>(sb, LDK, reinterpret_cast<const T*>(a.b) + offk, ldk, len, K);
  cp_tile32<kChunk, D, NTH>(sG, LDG, a.g + offk, ldk, len, K);
  cp_async_commit();
  cp_tile16<T, kChunk, D, NTH>(sv, LDK, reinterpret_cast<const T*>(a.v) + offv, ldv, len, V);
  cp_tile16<T, kChunk, D, NTH>(sw, LDK, reinterpret_cast<const T*>(a.w) + offv, ldv, len, V);
  cp_async_commit();
  for (int i = tid; i < kChunk * LDF; i += NTH) sAkk[i] = 0.f;
  if (tid == 0) sFlag[0] = 1;
  cp_async_wait<1>();
  __syncthreads();
  col_scan64_t<D, NTH, false>(sG, LDG, reinterpret_cast<float*>(R + L::rQs));
  for (int i = tid; i < kChunk * D; i += NTH) {
    const int r = i / D, cc = i - r * D;
    sG[r * LDG + cc] *= kLog2e;
  }
  for (int r = warp; r < kChunk; r += NTH / 32) {
    float s1 = 0.f, s2 = 0.f;
    for (int cc = lane; cc < D; cc += 32) {
      const float x = to_f<T>(sq[r * LDK + cc]), y = to_f<T>(sk[r * LDK + cc]);
      s1 += x * x;
      s2 += y * y;
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    if (lane == 0) {
      rq[r] = a.l2norm ? rsqrtf(s1 + kNormEps) : 1.f;
      rk[r] = a.l2norm ? rsqrtf(s2 + kNormEps) : 1.f;
    }
  }
  __syncthreads();

  // ---- Qg, Kd, gl out; score operands -----------------------------------------
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  T* gQg = reinterpret_cast<T*>(a.saved + a.L.qg) + ch * tileK;
  T* gKd = reinterpret_cast<T*>(a.saved + a.L.kd) + ch * tileK;
  float* gGl = reinterpret_cast<float*>(a.saved + a.L.gl) + ch * K;
  for (int i = tid; i < kChunk * (D / 2); i += NTH) {
    const int r = i / (D / 2), cc = (i - r * (D / 2)) * 2;
    const int rb = r & ~15;
    float qg[2], kd[2], qs[2], kbs[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float G = sG[r * LDG + cc + t], GL = sG[(kChunk - 1) * LDG + cc + t];
      const float qn = to_f<T>(sq[r * LDK + cc + t]) * rq[r];
      const float kn = to_f<T>(sk[r * LDK + cc + t]) * rk[r];
      const float f = exp2f(G - sG[rb * LDG + cc + t]);
      qg[t] = scale * qn * exp2f(G);
      kd[t] = kn * exp2f(GL - G);
      qs[t] = scale * qn * f;
      kbs[t] = to_f<T>(sb[r * LDK + cc + t]) * kn * f;
    }
    if (cc < K) {
      *reinterpret_cast<uint32_t*>(gQg + r * K + cc) = pack2<T>(qg[0], qg[1]);
      *reinterpret_cast<uint32_t*>(gKd + r * K + cc) = pack2<T>(kd[0], kd[1]);
    }
    *reinterpret_cast<uint32_t*>(sQs + r * LDK + cc) = pack2<T>(qs[0], qs[1]);
    *reinterpret_cast<uint32_t*>(sKBs + r * LDK + cc) = pack2<T>(kbs[0], kbs[1]);
  }
  for (int i = tid; i < K; i += NTH) gGl[i] = exp2f(sG[(kChunk - 1) * LDG + i]);
  for (int i = tid; i < 160 * (D / 2); i += NTH) {
    const int row = i / (D / 2), cc = (i - row * (D / 2)) * 2;
    const int I = row < 16 ? 0 : row < 48 ? 1 : row < 96 ? 2 : 3;
    const int r = row - 8 * I * (I + 1), r0 = 16 * I;
    float k2[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      const float e = fminf(sG[r0 * LDG + cc + t] - sG[r * LDG + cc + t], 120.f);
      k2[t] = to_f<T>(sk[r * LDK + cc + t]) * rk[r] * exp2f(e);
    }
    *reinterpret_cast<uint32_t*>(sKs + row * LDK + cc) = pack2<T>(k2[0], k2[1]);
  }
  for (int i = tid; i < 4 * D; i += NTH) {
    const int bI = i / D, cc = i - bI * D;
    const float rng = sG[(16 * bI) * LDG + cc] - sG[(16 * bI + 15) * LDG + cc];
    if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
  }
  __syncthreads();
  const bool safe = sFlag[0] != 0;

  // ---- score blocks: warp (I = wr, column block wc <= I) -------------------------
  T* gAqk = reinterpret_cast<T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk;
  {
    const int I = wr, J = wc;
    if (J <= I && (safe || J < I)) {
      const T* KsI = sKs + 8 * I * (I + 1) * LDK;
      float aq[1][2][4], ak[1][2][4];
      acc_zero(aq);
      acc_zero(ak);
      warp_mma16<1, 2, true, true>(aq, sQs, LDK, 16 * I, KsI, LDK, 16 * J, D);
      warp_mma16<1, 2, true, true>(ak, sKBs, LDK, 16 * I, KsI, LDK, 16 * J, D);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * I + gid + 8 * hf, i0 = 16 * J + 8 * j + 2 * tig;
          float x0 = aq[0][j][2 * hf], x1 = aq[0][j][2 * hf + 1];
          x0 = (i0 <= r) ? x0 : 0.f;
          x1 = (i0 + 1 <= r) ? x1 : 0.f;
          *reinterpret_cast<uint32_t*>(gAqk + r * kChunk + i0) = pack2<T>(x0, x1);
          sAkk[r * LDF + i0] = (i0 < r) ? ak[0][j][2 * hf] : 0.f;
          sAkk[r * LDF + i0 + 1] = (i0 + 1 < r) ? ak[0][j][2 * hf + 1] : 0.f;
        }
    } else if (J > I) {
      // strictly upper block: zeros
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * I + gid + 8 * hf, i0 = 16 * J + 8 * j + 2 * tig;
          *reinterpret_cast<uint32_t*>(gAqk + r * kChunk + i0) = pack2<T>(0.f, 0.f);
        }
    }
  }
  if (!safe) {
    // exact diagonal blocks: 2^(G_r - G_i) per element
    for (int idx = tid; idx < 4 * 256; idx += NTH) {
      const int bI = idx >> 8, e = idx & 255, rr = e >> 4, ii = e & 15;
      const int r = 16 * bI + rr, i = 16 * bI + ii;
      float sqv = 0.f, skv = 0.f;
      if (ii <= rr) {
        for (int cc = 0; cc < D; ++cc) {
          const float f = exp2f(sG[r * LDG + cc] - sG[i * LDG + cc]) *
                          to_f<T>(sk[i * LDK + cc]) * rk[i];
          sqv += to_f<T>(sq[r * LDK + cc]) * f;
          skv += to_f<T>(sb[r * LDK + cc]) * to_f<T>(sk[r * LDK + cc]) * f;
        }
        sqv *= scale * rq[r];
        skv *= rk[r];
      }
      gAqk[r * kChunk + i] = from_f<T>(sqv);
      sAkk[r * LDF + i] = (ii < rr) ? skv : 0.f;
    }
  }
  __syncthreads();

  // ---- A = (I + Akk)^-1 ----------------------------------------------------------
  float* sInv = reinterpret_cast<float*>(R + L::rInv);
  unit_lower_inverse<LDF>(sAkk, sInv, reinterpret_cast<float*>(R + L::rTmp));
  T* sA16 = reinterpret_cast<T*>(R + L::rA16);
  T* sE = reinterpret_cast<T*>(R + L::rE);
  T* sZ = reinterpret_cast<T*>(R + L::rZ);
  T* gA = reinterpret_cast<T*>(a.saved + a.L.a) + ch * kChunk * kChunk;
  for (int i = tid; i < kChunk * 32; i += NTH) {
    const int r = i >> 5, cc = (i & 31) * 2;
    const uint32_t pk = pack2<T>(sInv[r * LDF + cc], sInv[r * LDF + cc + 1]);
    *reinterpret_cast<uint32_t*>(sA16 + r * LDC + cc) = pk;
    *reinterpret_cast<uint32_t*>(gA + r * kChunk + cc) = pk;
  }
  cp_async_wait<0>();  // v, w
  __syncthreads();
  for (int i = tid; i < kChunk * (D / 2); i += NTH) {
    const int r = i / (D / 2), cc = (i - r * (D / 2)) * 2;
    float e2[2], z2[2];
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      e2[t] = to_f<T>(sb[r * LDK + cc + t]) * to_f<T>(sk[r * LDK + cc + t]) * rk[r] *
              exp2f(sG[r * LDG + cc + t]);
      z2[t] = to_f<T>(sv[r * LDK + cc + t]) * to_f<T>(sw[r * LDK + cc + t]);
    }
    *reinterpret_cast<uint32_t*>(sE + r * LDK + cc) = pack2<T>(e2[0], e2[1]);
    *reinterpret_cast<uint32_t*>(sZ + r * LDK + cc) = pack2<T>(z2[0], z2[1]);
  }
  __syncthreads();

  // ---- W = A E, U = A Z (owner tiles 16 x D/4) -----------------------------------
  {
    T* gW = reinterpret_cast<T*>(a.saved + a.L.w) + ch * tileK;
    T* gU = reinterpret_cast<T*>(a.saved + a.L.u) + ch * tileV;
    float acc[1][NTO][4];
    acc_zero(acc);
    warp_mma16<1, NTO, true, false>(acc, sA16, LDC, 16 * wr, sE, LDK, wc * DQ, kChunk);
#pragma unroll
    for (int j = 0; j < NTO; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
        if (cl < K)
          *reinterpret_cast<uint32_t*>(gW + r * K + cl) =
              pack2<T>(acc[0][j][2 * hf], acc[0][j][2 * hf + 1]);
      }
    acc_zero(acc);
    warp_mma16<1, NTO, true, false>(acc, sA16, LDC, 16 * wr, sZ, LDK, wc * DQ, kChunk);
#pragma unroll
    for (int j = 0; j < NTO; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
        if (cl < V)
          *reinterpret_cast<uint32_t*>(gU + r * V + cl) =
              pack2<T>(acc[0][j][2 * hf], acc[0][j][2 * hf + 1]);
      }
  }
}

template <typename T, int D>
cudaError_t launch_fwd_intra16(const FwdIntraArgs& a, cudaStream_t st) {
  auto kern = k_fwd_intra16<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Fwd16Layout<D>::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(a.seqs.n_chunks, a.H);
  kern<<<grid, kThreadsF16, Fwd16Layout<D>::bytes, st>>>(a);
  return cudaGetLastError();
}

template cudaError_t launch_fwd_intra16<__nv_bfloat16, 64>(const FwdIntraArgs&, cudaStream_t);
template cudaError_t launch_fwd_intra16<__nv_bfloat16, 128>(const FwdIntraArgs&, cudaStream_t);

}  // namespace gdn2
