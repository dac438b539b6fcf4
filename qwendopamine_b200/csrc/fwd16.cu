// fwd16.cu -- intra-chunk forward solve for bf16 inputs.
//
// One CTA of 16 warps per (chunk, head); same mathematics as k_fwd_intra
// (chunk_fwd.cu).  One cp.async round trip brings q, k, b, v, w and g.  After
// the decay scan and the row norms, a single elementwise pass writes Qg and
// Kd, forms E = b k_n 2^G and Z = v w in place of w and v, and builds the
// 16-bit score operands with per-16-row-block references
//   Qs[r] = scale q_n[r] 2^(G_r - G_b(r)),  KBs[r] = (b k_n)[r] 2^(G_r - G_b(r)),
//   Kb[i] = k_n[i] 2^(G_e(i) - G_i)
// (b(r) / e(i): first / last row of the row's block).  Every factor is <= 1.
// Block (I, J) of the scores uses the keys of block J scaled by
// 2^(G_16I - G_(16J+15)) while their fragments are loaded, so every product
// carries exactly 2^(G_r - G_i).  The scores, W = A E and U = A Z are
// mma.sync m16n8k16 products from ldmatrix fragments; the unit-lower inverse
// A = (I+Akk)^-1 stays in fp32 (register substitution for the diagonal
// blocks, 3-pass TF32 products for the rest).  Diagonal blocks whose 16-row
// decay range exceeds the fp32 exponent budget are recomputed elementwise.
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
  static constexpr int tile16 = kChunk * LDK * 2;
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + tile16;
  static constexpr int oB = oK + tile16;
  static constexpr int oV = oB + tile16;  // v, then Z = v * w
  static constexpr int oW = oV + tile16;  // w, then E = b k_n 2^G
  static constexpr int oG = oW + tile16;
  static constexpr int oMisc = oG + kChunk * LDG * 4;
  // misc floats: rq[64] rk[64] flag[4] Pb[4][D] Qe[4][D] F[10][D]
  static constexpr int nMisc = 64 + 64 + 4 + 18 * D;
  static constexpr int oR = oMisc + nMisc * 4;  // work region
  // scores
  static constexpr int rQs = 0;
  static constexpr int rKBs = rQs + tile16;
  static constexpr int rKb = rKBs + tile16;
  static constexpr int rAkk = rKb + tile16;
  static constexpr int rEndScores = rAkk + kChunk * LDF * 4;
  // inverse (reads Akk; Inv and the T tiles reuse the dead Qs / KBs / Kb)
  static constexpr int rInv = 0;
  static constexpr int rT = rInv + kChunk * LDF * 4;
  static constexpr int rA16 = rT + 3 * 16 * 20 * 4;  // written after the inverse
  static constexpr int rEndInv = rA16 + kChunk * LDC * 2;
  static constexpr int R = rEndScores > rEndInv ? rEndScores : rEndInv;
  static constexpr size_t bytes = (size_t)oR + R;
  static_assert(rT + 3 * 16 * 20 * 4 <= rAkk, "T tiles overlap Akk");
  // W / U staging: W over the dead Inv / T tiles below sA16, U past sA16
  static_assert(tile16 <= rA16 && rEndInv + tile16 <= R, "W / U staging tiles");
  static_assert(oR % 16 == 0 && rAkk % 16 == 0 && rA16 % 16 == 0, "alignment");
};

// acc_q / acc_k (16 x 16) += A_q / A_k (16 rows at m0, D columns) times the
// 16 key rows at n0 of Kb (K-major), each key column c scaled by F[c].
template <typename T, int D>
__device__ __forceinline__ void score_block16(float (&aq)[1][2][4], float (&ak)[1][2][4],
                                              const T* Aq, const T* Ak, int lda, int m0,
                                              const T* Kb, int n0, const float* F) {
  const int tig = threadIdx.x & 3;
#pragma unroll
  for (int k0 = 0; k0 < D; k0 += 16) {
    uint32_t a1[4], a2[4], b[4];
    load_a16<true>(a1, Aq, lda, m0, k0);
    load_a16<true>(a2, Ak, lda, m0, k0);
    load_b16x2<true>(b, Kb, lda, k0, n0);
    const float2 f0 = *reinterpret_cast<const float2*>(F + k0 + 2 * tig);
    const float2 f1 = *reinterpret_cast<const float2*>(F + k0 + 8 + 2 * tig);
    b[0] = scale_pair<T>(b[0], f0);
    b[1] = scale_pair<T>(b[1], f1);
    b[2] = scale_pair<T>(b[2], f0);
    b[3] = scale_pair<T>(b[3], f1);
    Mma16<T>::run(aq[0][0], a1, b[0], b[1]);
    Mma16<T>::run(aq[0][1], a1, b[2], b[3]);
    Mma16<T>::run(ak[0][0], a2, b[0], b[1]);
    Mma16<T>::run(ak[0][1], a2, b[2], b[3]);
  }
}

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
  float* sPb = rk + 64 + 4;  // [4][D]  2^G at each block's first row
  float* sQe = sPb + 4 * D;  // [4][D]  2^(G_63 - G) at each block's last row
  float* sF = sQe + 4 * D;   // [10][D] 2^(G_16I - G_(16J+15)), pair I(I+1)/2 + J
  unsigned char* R = sm + L::oR;
  T* sQs = reinterpret_cast<T*>(R + L::rQs);
  T* sKBs = reinterpret_cast<T*>(R + L::rKBs);
  T* sKb = reinterpret_cast<T*>(R + L::rKb);
  float* sAkk = reinterpret_cast<float*>(R + L::rAkk);
  float* sInv = reinterpret_cast<float*>(R + L::rInv);
  T* sA16 = reinterpret_cast<T*>(R + L::rA16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int wr = warp & 3, wc = warp >> 2;
  const int H = a.H, K = a.K, V = a.V;
  const int64_t ldk = (int64_t)H * K, ldv = (int64_t)H * V;
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const float scale = a.scale;
  const int n_items = a.seqs.n_chunks * H;

  // Items (chunk c, head h) = (item / H, item % H), strided over the grid.
  // q, k, b, g of the next item stream in (cp.async) once this item's scores
  // are done (they are dead from there on); v, w once its W / U products are.
  auto issue_qkbg = [&](int item) {
    const int c = item / H, h = item - (item / H) * H;
    const ChunkPos cp = chunk_pos(a.seqs, c);
    const int64_t offk = cp.row0 * ldk + (int64_t)h * K;
    cp_tile16<T, kChunk, D, NTH>(sq, LDK, reinterpret_cast<const T*>(a.q) + offk, ldk, cp.len, K);
    cp_tile16<T, kChunk, D, NTH>(sk, LDK, reinterpret_cast<const T*>(a.k) + offk, ldk, cp.len, K);
    cp_tile16<T, kChunk, D, NTH>(sb, LDK, reinterpret_cast<const T*>(a.b) + offk, ldk, cp.len, K);
    cp_tile32<kChunk, D, NTH>(sG, LDG, a.g + offk, ldk, cp.len, K);
    cp_async_commit();
  };
  auto issue_vw = [&](int item) {
    const int c = item / H, h = item - (item / H) * H;
    const ChunkPos cp = chunk_pos(a.seqs, c);
    const int64_t offv = cp.row0 * ldv + (int64_t)h * V;
    cp_tile16<T, kChunk, D, NTH>(sv, LDK, reinterpret_cast<const T*>(a.v) + offv, ldv, cp.len, V);
    cp_tile16<T, kChunk, D, NTH>(sw, LDK, reinterpret_cast<const T*>(a.w) + offv, ldv, cp.len, V);
    cp_async_commit();
  };
  issue_qkbg(blockIdx.x);
  issue_vw(blockIdx.x);

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int next = item + gridDim.x;
    const int c = item / H, h = item - (item / H) * H;
    const size_t ch = (size_t)c * H + h;
    if (tid == 0) sFlag[0] = 1;
    cp_async_wait<1>();  // q, k, b, g of this item
    __syncthreads();
    // chunk-local log2 cumulative decay
    col_scan64_reg<D, NTH, false>(sG, LDG, reinterpret_cast<float*>(R), kLog2e);
    // row norms: warp w owns rows 4w .. 4w+3
    {
      constexpr int EPL = D / 32;
      float s1[4], s2[4];
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const int r = 4 * warp + rr;
        s1[rr] = 0.f;
        s2[rr] = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float x = to_f<T>(sq[r * LDK + EPL * lane + e]);
          const float y = to_f<T>(sk[r * LDK + EPL * lane + e]);
          s1[rr] += x * x;
          s2[rr] += y * y;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          s1[rr] += __shfl_xor_sync(0xffffffffu, s1[rr], o);
          s2[rr] += __shfl_xor_sync(0xffffffffu, s2[rr], o);
        }
      if (lane < 4) {
        const int r = 4 * warp + lane;
        const float x1 = lane == 0 ? s1[0] : lane == 1 ? s1[1] : lane == 2 ? s1[2] : s1[3];
        const float x2 = lane == 0 ? s2[0] : lane == 1 ? s2[1] : lane == 2 ? s2[2] : s2[3];
        rq[r] = a.l2norm ? rsqrtf(x1 + kNormEps) : 1.f;
        rk[r] = a.l2norm ? rsqrtf(x2 + kNormEps) : 1.f;
      }
    }
    // per-block decay factors, diagonal-block safety, gl out
    float* gGl = reinterpret_cast<float*>(a.saved + a.L.gl) + ch * K;
    for (int i = tid; i < 18 * D; i += NTH) {
      const int p = i / D, cc = i - p * D;
      const float GL = sG[(kChunk - 1) * LDG + cc];
      float x;
      if (p < 4) {
        x = exp2f(sG[16 * p * LDG + cc]);
      } else if (p < 8) {
        x = exp2f(GL - sG[(16 * (p - 4) + 15) * LDG + cc]);
      } else {
        const int q = p - 8;
        const int I = q >= 6 ? 3 : q >= 3 ? 2 : q >= 1 ? 1 : 0;
        const int J = q - I * (I + 1) / 2;
        x = exp2f(fminf(sG[16 * I * LDG + cc] - sG[(16 * J + 15) * LDG + cc], 120.f));
      }
      sPb[i] = x;  // sPb, sQe, sF are contiguous
    }
    for (int i = tid; i < 4 * D; i += NTH) {
      const int bI = i / D, cc = i - bI * D;
      const float rng = sG[(16 * bI) * LDG + cc] - sG[(16 * bI + 15) * LDG + cc];
      if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
    }
    for (int i = tid; i < K; i += NTH) gGl[i] = exp2f(sG[(kChunk - 1) * LDG + i]);
    cp_async_wait<0>();  // v, w
    __syncthreads();
    const bool safe = sFlag[0] != 0;

    // ---- one elementwise pass: Qg, Kd out; Qs, KBs, Kb score operands;
    //      E = b k_n 2^G over w, Z = v w over v.  Thread = one column pair
    //      over RPT consecutive rows (all in one 16-row block).
    {
      constexpr int NCP = D / 2;               // column pairs
      constexpr int RPT = kChunk * NCP / NTH;  // rows per thread
      static_assert(RPT * NTH == kChunk * NCP && 16 % RPT == 0, "fused pass shape");
      const int cc = 2 * (tid % NCP), r0 = (tid / NCP) * RPT;
      const int blk = r0 >> 4, rb = r0 & ~15, re = rb + 15;
      T* gQg = reinterpret_cast<T*>(a.saved + a.L.qg) + ch * tileK;
      T* gKd = reinterpret_cast<T*>(a.saved + a.L.kd) + ch * tileK;
      const float2 Gb = *reinterpret_cast<const float2*>(sG + rb * LDG + cc);
      const float2 Ge = *reinterpret_cast<const float2*>(sG + re * LDG + cc);
      const float2 Pb = *reinterpret_cast<const float2*>(sPb + blk * D + cc);
      const float2 Qe = *reinterpret_cast<const float2*>(sQe + blk * D + cc);
#pragma unroll 4
      for (int j = 0; j < RPT; ++j) {
        const int r = r0 + j;
        const float2 G = *reinterpret_cast<const float2*>(sG + r * LDG + cc);
        const uint32_t uq = *reinterpret_cast<const uint32_t*>(sq + r * LDK + cc);
        const uint32_t uk = *reinterpret_cast<const uint32_t*>(sk + r * LDK + cc);
        const uint32_t ub = *reinterpret_cast<const uint32_t*>(sb + r * LDK + cc);
        const uint32_t uv = *reinterpret_cast<const uint32_t*>(sv + r * LDK + cc);
        const uint32_t uw = *reinterpret_cast<const uint32_t*>(sw + r * LDK + cc);
        const T* pq = reinterpret_cast<const T*>(&uq);
        const T* pk = reinterpret_cast<const T*>(&uk);
        const T* pb = reinterpret_cast<const T*>(&ub);
        const T* pv = reinterpret_cast<const T*>(&uv);
        const T* pw = reinterpret_cast<const T*>(&uw);
        const float nq = rq[r], nk = rk[r];
        const float g2[2] = {G.x, G.y}, gb2[2] = {Gb.x, Gb.y}, ge2[2] = {Ge.x, Ge.y};
        const float pb2[2] = {Pb.x, Pb.y}, qe2[2] = {Qe.x, Qe.y};
        float qg[2], kd[2], qs[2], kbs[2], kb[2], e2[2], z2[2];
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const float f = exp2f(g2[t] - gb2[t]);   // <= 1
          const float fe = exp2f(ge2[t] - g2[t]);  // <= 1
          const float qn = to_f<T>(pq[t]) * nq;
          const float kn = to_f<T>(pk[t]) * nk;
          const float bkn = to_f<T>(pb[t]) * kn;
          const float eG = pb2[t] * f;   // 2^G
          const float eK = qe2[t] * fe;  // 2^(G_63 - G)
          qg[t] = scale * qn * eG;
          kd[t] = kn * eK;
          qs[t] = scale * qn * f;
          kbs[t] = bkn * f;
          kb[t] = kn * fe;
          e2[t] = bkn * eG;
          z2[t] = to_f<T>(pv[t]) * to_f<T>(pw[t]);
        }
        if (cc < K) {
          *reinterpret_cast<uint32_t*>(gQg + r * K + cc) = pack2<T>(qg[0], qg[1]);
          *reinterpret_cast<uint32_t*>(gKd + r * K + cc) = pack2<T>(kd[0], kd[1]);
        }
        *reinterpret_cast<uint32_t*>(sQs + r * LDK + cc) = pack2<T>(qs[0], qs[1]);
        *reinterpret_cast<uint32_t*>(sKBs + r * LDK + cc) = pack2<T>(kbs[0], kbs[1]);
        *reinterpret_cast<uint32_t*>(sKb + r * LDK + cc) = pack2<T>(kb[0], kb[1]);
        *reinterpret_cast<uint32_t*>(sw + r * LDK + cc) = pack2<T>(e2[0], e2[1]);
        *reinterpret_cast<uint32_t*>(sv + r * LDK + cc) = pack2<T>(z2[0], z2[1]);
      }
    }
    __syncthreads();

    // ---- score blocks: warp (I = wr, column block J = wc <= I) --------------------
    // key i of block J enters block row I as Kb[i] 2^(G_16I - G_(16J+15)), so
    // every product carries exactly 2^(G_r - G_i).
    T* gAqk = reinterpret_cast<T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk;
    {
      const int I = wr, J = wc;
      if (J <= I && (safe || J < I)) {
        float aq[1][2][4], ak[1][2][4];
        acc_zero(aq);
        acc_zero(ak);
        score_block16<T, D>(aq, ak, sQs, sKBs, LDK, 16 * I, sKb, 16 * J,
                            sF + (I * (I + 1) / 2 + J) * D);
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
    if (next < n_items) issue_qkbg(next);  // q, k, b, g are dead for this item

    // ---- A = (I + Akk)^-1 ----------------------------------------------------------
    unit_lower_inverse_mma<LDF>(sAkk, sInv, reinterpret_cast<float*>(R + L::rT));
    T* gA = reinterpret_cast<T*>(a.saved + a.L.a) + ch * kChunk * kChunk;
    for (int i = tid; i < kChunk * 32; i += NTH) {
      const int r = i >> 5, cc = (i & 31) * 2;
      const uint32_t pk =
          (cc >> 4) <= (r >> 4) ? pack2<T>(sInv[r * LDF + cc], sInv[r * LDF + cc + 1]) : 0u;
      *reinterpret_cast<uint32_t*>(sA16 + r * LDC + cc) = pk;
      *reinterpret_cast<uint32_t*>(gA + r * kChunk + cc) = pk;
    }
    __syncthreads();

    // ---- W = A E, U = A Z (owner tiles 16 x D/4), staged for coalesced stores
    {
      T* stW = reinterpret_cast<T*>(R + L::rInv);  // Inv is dead after the pack
      T* stU = reinterpret_cast<T*>(R + L::rEndInv);  // past sA16 (read by both products)
      float acc[1][NTO][4];
      acc_zero(acc);
      warp_mma16<1, NTO, true, false>(acc, sA16, LDC, 16 * wr, sw, LDK, wc * DQ, kChunk);
#pragma unroll
      for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
          *reinterpret_cast<uint32_t*>(stW + r * LDK + cl) =
              pack2<T>(acc[0][j][2 * hf], acc[0][j][2 * hf + 1]);
        }
      acc_zero(acc);
      warp_mma16<1, NTO, true, false>(acc, sA16, LDC, 16 * wr, sv, LDK, wc * DQ, kChunk);
#pragma unroll
      for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
          *reinterpret_cast<uint32_t*>(stU + r * LDK + cl) =
              pack2<T>(acc[0][j][2 * hf], acc[0][j][2 * hf + 1]);
        }
      __syncthreads();
      store_tile16<T, kChunk, D, NTH>(reinterpret_cast<T*>(a.saved + a.L.w) + ch * tileK, K, stW,
                                      LDK, kChunk, K);
      store_tile16<T, kChunk, D, NTH>(reinterpret_cast<T*>(a.saved + a.L.u) + ch * tileV, V, stU,
                                      LDK, kChunk, V);
    }
    __syncthreads();
    if (next < n_items) issue_vw(next);  // v, w (now E, Z) are dead
  }
  cp_async_wait<0>();
}

template <typename T, int D>
cudaError_t launch_fwd_intra16(const FwdIntraArgs& a, cudaStream_t st) {
  auto kern = k_fwd_intra16<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Fwd16Layout<D>::bytes);
  if (e != cudaSuccess) return e;
  const int n_items = a.seqs.n_chunks * a.H;
  if (n_items == 0) return cudaSuccess;
  int sms = 0;
  e = num_sms(&sms);
  if (e != cudaSuccess) return e;
  const int grid = n_items < sms ? n_items : sms;  // persistent: one CTA per SM
  kern<<<grid, kThreadsF16, Fwd16Layout<D>::bytes, st>>>(a);
  return cudaGetLastError();
}

template cudaError_t launch_fwd_intra16<__nv_bfloat16, 64>(const FwdIntraArgs&, cudaStream_t);
template cudaError_t launch_fwd_intra16<__nv_bfloat16, 128>(const FwdIntraArgs&, cudaStream_t);

}  // namespace gdn2
