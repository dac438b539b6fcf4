// fwd16.cu -- intra-chunk forward solve for bf16 inputs.
//
// Persistent: one CTA of 16 warps per SM walks (chunk, head) items; same
// mathematics as k_fwd_intra (chunk_fwd.cu).  q, k, b, g and v, w arrive as
// TMA boxes (128-byte swizzled, read through swz<>) requested by one thread
// for the next item as soon as the current item is done with them.  After
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
// blocks, TF32 products for the rest, as the reference's solve does).  Diagonal blocks whose 16-row
// decay range exceeds the fp32 exponent budget are recomputed elementwise.
#include "chunk_args.cuh"
#include "inverse.cuh"
#include "mma16.cuh"
#include "tc.cuh"

namespace gdn2 {

constexpr int kThreadsF16 = 512;

// Byte offset of element (r, c) of a 64-row tile of EB-byte elements stored
// as TMA boxes of 128 bytes x 64 rows with the 128-byte swizzle (box b holds
// bytes [128 b, 128 b + 128) of every row; 16-byte chunks XOR-ed with r % 8).
template <int EB>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  const uint32_t byte = (uint32_t)c * EB;
  return (byte >> 7) * 8192u + (uint32_t)r * 128u + ((((byte >> 4) & 7u) ^ (uint32_t)(r & 7)) << 4) +
         (byte & 15u);
}

template <int D>
struct Fwd16Layout {
  static constexpr int LDK = D + 8;        // padded 16-bit work tiles
  static constexpr int LDC = kChunk + 8;   // 16-bit 64 x 64
  static constexpr int LDF = kChunk + 4;   // fp32 64 x 64
  static constexpr int tile16 = kChunk * LDK * 2;
  static constexpr int sw16 = (D / 64) * 8192;  // swizzled bf16 [64][D] (TMA)
  static constexpr int swG = (D / 32) * 8192;   // swizzled fp32 [64][D] (TMA)
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + sw16;
  static constexpr int oB = oK + sw16;
  static constexpr int oV = oB + sw16;  // v, then Z = v * w
  static constexpr int oW = oV + sw16;  // w, then E = b k_n 2^G
  static constexpr int oG = oW + sw16;
  static constexpr int oMisc = oG + swG;
  // misc floats: rq[64] rk[64] flag[4] Pb[4][D] Qe[4][D] F[10][D] mbar[2] (as 4)
  static constexpr int nMisc = 64 + 64 + 4 + 18 * D + 4;
  static constexpr int oR = (oMisc + nMisc * 4 + 15) / 16 * 16;  // work region
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
  static constexpr size_t bytes = (size_t)oR + R + 1024;  // + alignment slack
  static_assert(rT + 3 * 16 * 20 * 4 <= rAkk, "T tiles overlap Akk");
  // W / U staging: W over the dead Inv / T tiles below sA16, U past sA16
  static_assert(tile16 <= rA16 && rEndInv + tile16 <= R, "W / U staging tiles");
  static_assert(rAkk % 16 == 0 && rA16 % 16 == 0, "alignment");
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

// acc1 += A B1 and acc2 += A B2: A = 16 rows at m0 of a padded K-major tile
// (kd columns, its fragments loaded once), B1 / B2 = kd rows x 8*NT columns
// at n0 of swizzled [64][D] tiles.
template <int NT, typename T>
__device__ __forceinline__ void mma_a_swb2(float (&acc1)[1][NT][4], float (&acc2)[1][NT][4],
                                           const T* A, int lda, int m0, const unsigned char* B1,
                                           const unsigned char* B2, int n0, int kd) {
  const int lane = threadIdx.x & 31;
  const int j8 = lane >> 3, rr = lane & 7;
#pragma unroll
  for (int k0 = 0; k0 < kd; k0 += 16) {
    uint32_t a[4];
    load_a16<true>(a, A, lda, m0, k0);
#pragma unroll
    for (int j = 0; j < NT; j += 2) {
      uint32_t b[4];
      const int k = k0 + rr + ((j8 & 1) << 3), n = n0 + 8 * j + ((j8 >> 1) << 3);
      ldsm_x4_t(b, B1 + swz<2>(k, n));
      Mma16<T>::run(acc1[0][j], a, b[0], b[1]);
      Mma16<T>::run(acc1[0][j + 1], a, b[2], b[3]);
      ldsm_x4_t(b, B2 + swz<2>(k, n));
      Mma16<T>::run(acc2[0][j], a, b[0], b[1]);
      Mma16<T>::run(acc2[0][j + 1], a, b[2], b[3]);
    }
  }
}

// Inclusive prefix sum down the 64 rows of a swizzled fp32 tile, times mul
// (register-staged, same summation order as col_scan64_reg).
template <int NC, int NTH>
__device__ __forceinline__ void col_scan64_sw(unsigned char* s, float* tmp, float mul) {
  constexpr int NSEG = NTH / NC;
  constexpr int RPS = kChunk / NSEG;
  static_assert(NSEG * NC == NTH && RPS * NSEG == kChunk, "scan shape");
  const int col = threadIdx.x % NC, seg = threadIdx.x / NC;
  float x[RPS];
#pragma unroll
  for (int i = 0; i < RPS; ++i) x[i] = *reinterpret_cast<const float*>(s + swz<4>(seg * RPS + i, col));
#pragma unroll
  for (int i = 1; i < RPS; ++i) x[i] += x[i - 1];
  tmp[seg * NC + col] = x[RPS - 1];
  __syncthreads();
  float off = 0.f;
#pragma unroll
  for (int j = 0; j < NSEG - 1; ++j)
    if (j < seg) off += tmp[j * NC + col];
#pragma unroll
  for (int i = 0; i < RPS; ++i)
    *reinterpret_cast<float*>(s + swz<4>(seg * RPS + i, col)) = (x[i] + off) * mul;
  __syncthreads();
}

// The same scan for 128 columns (four 64-row segments of 16 rows: segment I
// is row block I), whose epilogue also writes the per-block decay factors
// from the values it stores (so they equal what a later read would give):
//   Pb[I] = 2^G_16I,  Qe[I] = 2^(G_63 - G_(16I+15)),
//   F[I(I+1)/2 + J] = 2^min(G_16I - G_(16J+15), 120)  (J <= I),
// clears *safe when block I's decay range exceeds kSafeLog2Range, and writes
// gl = 2^G_63 for the first K columns.
template <int NTH>
__device__ __forceinline__ void col_scan64_sw_factors(unsigned char* s, float* tmp, float mul,
                                                      float* sPb, float* sQe, float* sF,
                                                      int* safe, float* gl, int K) {
  constexpr int NC = 128, NSEG = NTH / NC, RPS = kChunk / NSEG;
  static_assert(NSEG == 4 && RPS == 16, "one 16-row block per segment");
  const int col = threadIdx.x % NC, I = threadIdx.x / NC;
  float x[RPS];
#pragma unroll
  for (int i = 0; i < RPS; ++i) x[i] = *reinterpret_cast<const float*>(s + swz<4>(I * RPS + i, col));
#pragma unroll
  for (int i = 1; i < RPS; ++i) x[i] += x[i - 1];
  tmp[I * NC + col] = x[RPS - 1];
  __syncthreads();
  float off[NSEG];  // off[j]: sum of the segment totals before segment j
  off[0] = 0.f;
#pragma unroll
  for (int j = 1; j < NSEG; ++j) off[j] = off[j - 1] + tmp[(j - 1) * NC + col];
  float o = 0.f;
#pragma unroll
  for (int j = 0; j < NSEG; ++j)
    if (j == I) o = off[j];
#pragma unroll
  for (int i = 0; i < RPS; ++i)
    *reinterpret_cast<float*>(s + swz<4>(I * RPS + i, col)) = (x[i] + o) * mul;
  float glast[NSEG];  // G at each block's last row, as stored
#pragma unroll
  for (int j = 0; j < NSEG; ++j) glast[j] = (tmp[j * NC + col] + off[j]) * mul;
  const float gfirst = (x[0] + o) * mul, GL = glast[NSEG - 1];
  float gl_I = glast[0];
#pragma unroll
  for (int j = 1; j < NSEG; ++j)
    if (j == I) gl_I = glast[j];
  sPb[I * NC + col] = fast_exp2(gfirst);
  sQe[I * NC + col] = fast_exp2(GL - gl_I);
#pragma unroll
  for (int J = 0; J < NSEG; ++J)
    if (J <= I) sF[(I * (I + 1) / 2 + J) * NC + col] = fast_exp2(fminf(gfirst - glast[J], 120.f));
  if (!(gfirst - gl_I <= kSafeLog2Range)) *safe = 0;
  if (I == NSEG - 1 && col < K) gl[col] = exp2f(GL);
  __syncthreads();
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreadsF16, 1)
    k_fwd_intra16(FwdIntraArgs a, const __grid_constant__ CUtensorMap mQ,
                  const __grid_constant__ CUtensorMap mK, const __grid_constant__ CUtensorMap mB,
                  const __grid_constant__ CUtensorMap mV, const __grid_constant__ CUtensorMap mW,
                  const __grid_constant__ CUtensorMap mG) {
  using L = Fwd16Layout<D>;
  constexpr int LDK = L::LDK, LDC = L::LDC, LDF = L::LDF;
  constexpr int NTH = kThreadsF16;
  constexpr int DQ = D / 4, NTO = DQ / 8;
  extern __shared__ unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  unsigned char* sq = sm + L::oQ;  // swizzled TMA tiles
  unsigned char* sk = sm + L::oK;
  unsigned char* sb = sm + L::oB;
  unsigned char* sv = sm + L::oV;
  unsigned char* sw = sm + L::oW;
  unsigned char* sG = sm + L::oG;
  float* rq = reinterpret_cast<float*>(sm + L::oMisc);
  float* rk = rq + 64;
  int* sFlag = reinterpret_cast<int*>(rk + 64);
  float* sPb = rk + 64 + 4;  // [4][D]  2^G at each block's first row
  float* sQe = sPb + 4 * D;  // [4][D]  2^(G_63 - G) at each block's last row
  float* sF = sQe + 4 * D;   // [10][D] 2^(G_16I - G_(16J+15)), pair I(I+1)/2 + J
  uint64_t* barA = reinterpret_cast<uint64_t*>(sF + 10 * D);  // q, k, b, g landed
  uint64_t* barB = barA + 1;                                  // v, w landed
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
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const float scale = a.scale;
  const int n_items = a.seqs.n_chunks * H;
  const int nbK = (K + 63) / 64, nbV = (V + 63) / 64, nbG = (K + 31) / 32;
  auto G_ = [&](int r, int c) -> float { return *reinterpret_cast<const float*>(sG + swz<4>(r, c)); };
  auto E16 = [&](const unsigned char* t, int r, int c) -> float {
    return to_f<T>(*reinterpret_cast<const T*>(t + swz<2>(r, c)));
  };

  // Items (chunk c, head h) = (item / H, item % H), strided over the grid.
  // Thread 0 requests each item's tiles as TMA boxes (3-D views [rows][H][D],
  // 64 rows x 128 bytes each) completing on an mbarrier: q, k, b, g of the
  // next item once this item's fused pass (or, with an exact diagonal block,
  // its scores) is done with them, v, w once its W / U products are done.
  // (row0 of the item's chunk comes from the sequence tables, looked up one
  // item ahead so the dependent global loads stay off the critical path)
  auto issue_qkbg = [&](int item, int row0) {
    const int h = item - (item / H) * H;
    tc::mbar_expect_tx(barA, (uint32_t)(3 * nbK + nbG) * 8192u);
    for (int bx = 0; bx < nbK; ++bx) {
      tc::tma_load_3d(sq + bx * 8192, &mQ, 64 * bx, h, row0, barA);
      tc::tma_load_3d(sk + bx * 8192, &mK, 64 * bx, h, row0, barA);
      tc::tma_load_3d(sb + bx * 8192, &mB, 64 * bx, h, row0, barA);
    }
    for (int bx = 0; bx < nbG; ++bx) tc::tma_load_3d(sG + bx * 8192, &mG, 32 * bx, h, row0, barA);
  };
  auto issue_vw = [&](int item, int row0) {
    const int h = item - (item / H) * H;
    tc::mbar_expect_tx(barB, (uint32_t)(2 * nbV) * 8192u);
    for (int bx = 0; bx < nbV; ++bx) {
      tc::tma_load_3d(sv + bx * 8192, &mV, 64 * bx, h, row0, barB);
      tc::tma_load_3d(sw + bx * 8192, &mW, 64 * bx, h, row0, barB);
    }
  };
  // rows past a partial chunk's end hold the next sequence's tokens
  auto zero_rows = [&](unsigned char* t, int nbox, int len) {
    for (int e = tid; e < (kChunk - len) * nbox * 8; e += NTH) {
      const int r = len + e / (nbox * 8), rest = e - (e / (nbox * 8)) * (nbox * 8);
      *reinterpret_cast<uint4*>(t + (rest >> 3) * 8192 + r * 128 + (rest & 7) * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // boxes past K / V are never loaded and stay zero
  for (int i = tid; i < (5 * L::sw16 + L::swG) / 16; i += NTH)
    reinterpret_cast<uint4*>(sm)[i] = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    tc::mbar_init(barA, 1);
    tc::mbar_init(barB, 1);
    tc::fence_mbar_init();
  }
  tc::fence_async_smem();
  __syncthreads();
  ChunkPos cur = chunk_pos(a.seqs, blockIdx.x / H);
  if (tid == 0) {
    issue_qkbg(blockIdx.x, (int)cur.row0);
    issue_vw(blockIdx.x, (int)cur.row0);
  }
  int fault = 0;
  uint32_t phase = 0;

  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int next = item + gridDim.x;
    const int c = item / H, h = item - (item / H) * H;
    const size_t ch = (size_t)c * H + h;
    const int len = cur.len;
    ChunkPos nxt = cur;
    if (next < n_items) nxt = chunk_pos(a.seqs, next / H);
    if (tid == 0) sFlag[0] = 1;
    if (!tc::mbar_wait(barA, phase)) fault = 1;  // q, k, b, g of this item
    if (__syncthreads_or(fault)) break;
    if (len < kChunk) {
      zero_rows(sq, nbK, len);
      zero_rows(sk, nbK, len);
      zero_rows(sb, nbK, len);
      zero_rows(sG, nbG, len);
      tc::fence_async_smem();
      __syncthreads();
    }
    if (a.gate.mode) {  // gate in kernel: raw input -> log-decay (valid rows / channels)
      for (int i = tid; i < kChunk * D; i += NTH) {
        const int r = i / D, cc = i - r * D;
        if (r < len && cc < K) {
          float* pg = reinterpret_cast<float*>(sG + swz<4>(r, cc));
          *pg = gate_apply(a.gate, *pg, h, cc, K);
        }
      }
      __syncthreads();
    }
    // chunk-local log2 cumulative decay (for 128 columns with the per-block
    // decay factors, diagonal-block safety and gl in the same pass)
    float* gGl = reinterpret_cast<float*>(a.saved + a.L.gl) + ch * K;
    if constexpr (D == 128)
      col_scan64_sw_factors<NTH>(sG, reinterpret_cast<float*>(R), kLog2e, sPb, sQe, sF, sFlag,
                                 gGl, K);
    else
      col_scan64_sw<D, NTH>(sG, reinterpret_cast<float*>(R), kLog2e);
    // row norms: warp w owns rows 4w .. 4w+3
    {
      constexpr int EPL = D / 32;
      float s1[4], s2[4];
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) {
        const int r = 4 * warp + rr;
        s1[rr] = 0.f;
        s2[rr] = 0.f;
        // the lane's EPL columns are contiguous inside one 16-byte chunk
        const uint32_t o = swz<2>(r, EPL * lane);
        uint32_t uq[EPL / 2], uk[EPL / 2];
        if constexpr (EPL == 4) {
          const uint2 x = *reinterpret_cast<const uint2*>(sq + o);
          const uint2 y = *reinterpret_cast<const uint2*>(sk + o);
          uq[0] = x.x; uq[1] = x.y; uk[0] = y.x; uk[1] = y.y;
        } else {
          uq[0] = *reinterpret_cast<const uint32_t*>(sq + o);
          uk[0] = *reinterpret_cast<const uint32_t*>(sk + o);
        }
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float x = to_f<T>(reinterpret_cast<const T*>(uq)[e]);
          const float y = to_f<T>(reinterpret_cast<const T*>(uk)[e]);
          s1[rr] += x * x;
          s2[rr] += y * y;
        }
      }
      const float v8[8] = {s1[0], s1[1], s1[2], s1[3], s2[0], s2[1], s2[2], s2[3]};
      const float tot = warp_reduce8(v8, lane);
      if ((lane & 3) == 0) {
        const int idx = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
        const int r = 4 * warp + (idx & 3);
        (idx < 4 ? rq : rk)[r] = a.l2norm ? rsqrtf(tot + kNormEps) : 1.f;
      }
    }
    // per-block decay factors, diagonal-block safety, gl out (64 columns)
    if constexpr (D != 128) {
    for (int i = tid; i < 18 * D; i += NTH) {
      const int p = i / D, cc = i - p * D;
      const float GL = G_(kChunk - 1, cc);
      float x;
      if (p < 4) {
        x = fast_exp2(G_(16 * p, cc));
      } else if (p < 8) {
        x = fast_exp2(GL - G_(16 * (p - 4) + 15, cc));
      } else {
        const int q = p - 8;
        const int I = q >= 6 ? 3 : q >= 3 ? 2 : q >= 1 ? 1 : 0;
        const int J = q - I * (I + 1) / 2;
        x = fast_exp2(fminf(G_(16 * I, cc) - G_(16 * J + 15, cc), 120.f));
      }
      sPb[i] = x;  // sPb, sQe, sF are contiguous
    }
    for (int i = tid; i < 4 * D; i += NTH) {
      const int bI = i / D, cc = i - bI * D;
      const float rng = G_(16 * bI, cc) - G_(16 * bI + 15, cc);
      if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
    }
    for (int i = tid; i < K; i += NTH) gGl[i] = exp2f(G_(kChunk - 1, i));
    }
    if (!tc::mbar_wait(barB, phase)) fault = 1;  // v, w
    if (__syncthreads_or(fault)) break;
    if (len < kChunk) {
      zero_rows(sv, nbV, len);
      zero_rows(sw, nbV, len);
      tc::fence_async_smem();
      __syncthreads();
    }
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
      const float2 Gb = *reinterpret_cast<const float2*>(sG + swz<4>(rb, cc));
      const float2 Ge = *reinterpret_cast<const float2*>(sG + swz<4>(re, cc));
      const float2 Pb = *reinterpret_cast<const float2*>(sPb + blk * D + cc);
      const float2 Qe = *reinterpret_cast<const float2*>(sQe + blk * D + cc);
#pragma unroll 4
      for (int j = 0; j < RPT; ++j) {
        const int r = r0 + j;
        const uint32_t o16 = swz<2>(r, cc);
        const float2 G = *reinterpret_cast<const float2*>(sG + swz<4>(r, cc));
        const uint32_t uq = *reinterpret_cast<const uint32_t*>(sq + o16);
        const uint32_t uk = *reinterpret_cast<const uint32_t*>(sk + o16);
        const uint32_t ub = *reinterpret_cast<const uint32_t*>(sb + o16);
        const uint32_t uv = *reinterpret_cast<const uint32_t*>(sv + o16);
        const uint32_t uw = *reinterpret_cast<const uint32_t*>(sw + o16);
        const float2 f = exp2_2(make_float2(G.x - Gb.x, G.y - Gb.y));   // <= 1
        const float2 fe = exp2_2(make_float2(Ge.x - G.x, Ge.y - G.y));  // <= 1
        const float2 qn = mul2(unpack2<T>(uq), f2(rq[r]));
        const float2 kn = mul2(unpack2<T>(uk), f2(rk[r]));
        const float2 bkn = mul2(unpack2<T>(ub), kn);
        const float2 eG = mul2(Pb, f);   // 2^G
        const float2 eK = mul2(Qe, fe);  // 2^(G_63 - G)
        const float2 sqn = mul2(f2(scale), qn);
        const float2 qg = mul2(sqn, eG), kd = mul2(kn, eK), qs = mul2(sqn, f);
        const float2 kbs = mul2(bkn, f), kb = mul2(kn, fe), e2 = mul2(bkn, eG);
        const float2 z2 = mul2(unpack2<T>(uv), unpack2<T>(uw));
        if (cc < K) {
          *reinterpret_cast<uint32_t*>(gQg + r * K + cc) = pack2<T>(qg.x, qg.y);
          *reinterpret_cast<uint32_t*>(gKd + r * K + cc) = pack2<T>(kd.x, kd.y);
        }
        *reinterpret_cast<uint32_t*>(sQs + r * LDK + cc) = pack2<T>(qs.x, qs.y);
        *reinterpret_cast<uint32_t*>(sKBs + r * LDK + cc) = pack2<T>(kbs.x, kbs.y);
        *reinterpret_cast<uint32_t*>(sKb + r * LDK + cc) = pack2<T>(kb.x, kb.y);
        *reinterpret_cast<uint32_t*>(sw + o16) = pack2<T>(e2.x, e2.y);
        *reinterpret_cast<uint32_t*>(sv + o16) = pack2<T>(z2.x, z2.y);
      }
    }
    tc::fence_async_smem();
    __syncthreads();
    // With safe diagonal blocks nothing reads q, k, b, g after the fused pass,
    // so the next item's copies start now (the exact diagonal path below
    // still reads them: then they start after the scores).
    if (safe && tid == 0 && next < n_items) issue_qkbg(next, (int)nxt.row0);

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
            const float f = exp2f(G_(r, cc) - G_(i, cc)) * E16(sk, i, cc) * rk[i];
            sqv += E16(sq, r, cc) * f;
            skv += E16(sb, r, cc) * E16(sk, r, cc) * f;
          }
          sqv *= scale * rq[r];
          skv *= rk[r];
        }
        gAqk[r * kChunk + i] = from_f<T>(sqv);
        sAkk[r * LDF + i] = (ii < rr) ? skv : 0.f;
      }
    }
    tc::fence_async_smem();
    __syncthreads();
    if (!safe && tid == 0 && next < n_items) issue_qkbg(next, (int)nxt.row0);  // now dead

    // ---- A = (I + Akk)^-1 ----------------------------------------------------------
    // (single-term TF32 products: A is stored in bf16 and feeds bf16 products,
    // and the reference's solve uses TF32 products here as well)
    unit_lower_inverse_mma<LDF, 1>(sAkk, sInv, reinterpret_cast<float*>(R + L::rT));
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
      T* stW = reinterpret_cast<T*>(R + L::rInv);     // Inv is dead after the pack
      T* stU = reinterpret_cast<T*>(R + L::rEndInv);  // past sA16 (read by both products)
      float accW[1][NTO][4], accU[1][NTO][4];
      acc_zero(accW);
      acc_zero(accU);
      mma_a_swb2<NTO, T>(accW, accU, sA16, LDC, 16 * wr, sw, sv, wc * DQ, kChunk);
#pragma unroll
      for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
          *reinterpret_cast<uint32_t*>(stW + r * LDK + cl) =
              pack2<T>(accW[0][j][2 * hf], accW[0][j][2 * hf + 1]);
          *reinterpret_cast<uint32_t*>(stU + r * LDK + cl) =
              pack2<T>(accU[0][j][2 * hf], accU[0][j][2 * hf + 1]);
        }
      tc::fence_async_smem();
      __syncthreads();
      if (tid == 0 && next < n_items) issue_vw(next, (int)nxt.row0);  // v, w (now E, Z) are dead
      store_tile16<T, kChunk, D, NTH>(reinterpret_cast<T*>(a.saved + a.L.w) + ch * tileK, K, stW,
                                      LDK, kChunk, K);
      store_tile16<T, kChunk, D, NTH>(reinterpret_cast<T*>(a.saved + a.L.u) + ch * tileV, V, stU,
                                      LDK, kChunk, V);
    }
    __syncthreads();
    phase ^= 1u;
    cur = nxt;
  }
  if (fault && tid == 0) {
    // a copy never landed: wait (bounded) for what is still in flight, flag it
    tc::mbar_wait(barA, phase);
    tc::mbar_wait(barB, phase);
    atomicOr(a.fault, 2u);
  }
}

template <typename T, int D>
cudaError_t launch_fwd_intra16(const FwdIntraArgs& a, cudaStream_t st) {
  auto kern = k_fwd_intra16<T, D>;
  const int n_items = a.seqs.n_chunks * a.H;
  if (n_items == 0) return cudaSuccess;
  const uint64_t rows = (uint64_t)a.total_rows, H = (uint64_t)a.H;
  CUtensorMap mQ, mK, mB, mV, mW, mG;
  if (!tmap_rows(&mQ, a.q, a.K, H, rows, 64, 2) || !tmap_rows(&mK, a.k, a.K, H, rows, 64, 2) ||
      !tmap_rows(&mB, a.b, a.K, H, rows, 64, 2) || !tmap_rows(&mV, a.v, a.V, H, rows, 64, 2) ||
      !tmap_rows(&mW, a.w, a.V, H, rows, 64, 2) || !tmap_rows(&mG, a.g, a.K, H, rows, 32, 4))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)Fwd16Layout<D>::bytes);
  if (e != cudaSuccess) return e;
  int sms = 0;
  e = num_sms(&sms);
  if (e != cudaSuccess) return e;
  // persistent: one CTA per SM, or fewer when the caller leaves SMs to a
  // state pass running beside this launch
  if (a.max_ctas > 0 && a.max_ctas < sms) sms = a.max_ctas;
  const int grid = n_items < sms ? n_items : sms;
  kern<<<grid, kThreadsF16, Fwd16Layout<D>::bytes, st>>>(a, mQ, mK, mB, mV, mW, mG);
  return cudaGetLastError();
}

template cudaError_t launch_fwd_intra16<__nv_bfloat16, 64>(const FwdIntraArgs&, cudaStream_t);
template cudaError_t launch_fwd_intra16<__nv_bfloat16, 128>(const FwdIntraArgs&, cudaStream_t);

}  // namespace gdn2
