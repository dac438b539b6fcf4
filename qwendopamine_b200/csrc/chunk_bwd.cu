// chunk_bwd.cu -- chunkwise GDN-2 backward on B200.
//
// Per chunk the forward computed (G: chunk-local cumulative log decay)
//   VN = U - W h,  o = Qg h + Aqk VN,  h' = gl*h + Kd^T VN,
//   U = A (w*v),  W = A E,  E = b*k*e^G,  A = (I + Akk)^-1,
//   Qg = scale*q*e^G,  Kd = k*e^(G_last - G),  gl = e^G_last.
//
// k_bwd_state: one CTA per (sequence, head, 32-column value tile), reverse
//   over the sequence's chunks (replaces K10, chunk_kda.py:1733-2213).  With
//   dh the gradient w.r.t. the state leaving the chunk:
//     dVN = Aqk^T dO + Kd dh;   dh <- gl*dh + Qg^T dO - W^T dVN.
//   dh (per chunk, before the update) and dVN are kept for the next kernel.
//
// k_bwd_intra: one CTA per (chunk, head), fully parallel (replaces K9, K11,
//   K12, K13 and FLA l2norm_bwd, chunk_gdn2.py:1437-2167).  Value side,
//   accumulated over 32-column value slices in registers:
//     dQg = dO h^T,  dKd = VN dh^T,  dW = -dVN h^T,  dgl = rowsum(h*dh),
//     dAqk = tril(dO VN^T),  dA = dVN (w*v)^T [+ dW E^T],  dZ = A^T dVN,
//     dv = dZ*w,  dw = dZ*v.
//   Key side, per 32-column key block:
//     dAkk = -tril_strict(A^T dA A^T),  dE = A^T dW,
//     score backward for Aqk and Akk with the same per-16-row reference rows
//     as the forward, then the chain through Qg, Kd, E, gl:
//     dG = q*dq + kb*dkb - k*dk_dir (+ dG_last on the last row),
//     dg = reverse cumsum of dG,  db = dkb*k,  dk = dk_dir + dkb*b,
//   and finally the l2norm backward on dq and dk.
#include "chunk_args.cuh"

namespace gdn2 {

template <int D>
struct BStateSmem {
  static constexpr int LD = D + 4;
  static constexpr int LDC = kChunk + 4;
  static constexpr int LDB = kBV + 4;
  static constexpr int floats = 3 * kChunk * LD + kChunk * LDC + 2 * kChunk * LDB + D * LDB + D;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) k_bwd_state(BwdStateArgs a) {
  using S = BStateSmem<D>;
  constexpr int LD = S::LD, LDC = S::LDC, LDB = S::LDB;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sQg = sm;
  float* sKd = sQg + kChunk * LD;
  float* sW = sKd + kChunk * LD;
  float* sAqk = sW + kChunk * LD;
  float* sDO = sAqk + kChunk * LDC;  // [64][LDB]
  float* sDVN = sDO + kChunk * LDB;  // [64][LDB]
  float* sDH = sDVN + kChunk * LDB;  // [D][LDB]
  float* sGl = sDH + D * LDB;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int H = a.H, K = a.K, V = a.V;
  const int nh = blockIdx.y, n = nh / H, h = nh - n * H;
  const int v0 = blockIdx.x * kBV;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];

  for (int idx = tid; idx < D * kBV; idx += blockDim.x) {
    int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
    float x = 0.f;
    if (a.dht && r < K && col < V) x = a.dht[(((int64_t)n * H + h) * K + r) * V + col];
    sDH[r * LDB + cc] = x;
  }
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const int64_t ldo = (int64_t)H * V;
  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 16;

  for (int c = c_end - 1; c >= c_begin; --c) {
    const size_t ch = (size_t)c * H + h;
    const ChunkPos cp = chunk_pos(a.seqs, c);
    load_tile<T, kChunk, D>(sQg, LD, reinterpret_cast<const T*>(a.saved + a.L.qg) + ch * tileK, K,
                            kChunk, K);
    load_tile<T, kChunk, D>(sKd, LD, reinterpret_cast<const T*>(a.saved + a.L.kd) + ch * tileK, K,
                            kChunk, K);
    load_tile<T, kChunk, D>(sW, LD, reinterpret_cast<const T*>(a.saved + a.L.w) + ch * tileK, K,
                            kChunk, K);
    load_tile<T, kChunk, kChunk>(sAqk, LDC,
                                 reinterpret_cast<const T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk,
                                 kChunk, kChunk, kChunk);
    const T* gdo = reinterpret_cast<const T*>(a.dout) + cp.row0 * ldo + (int64_t)h * V + v0;
    load_tile<T, kChunk, kBV>(sDO, LDB, gdo, ldo, cp.len, min(kBV, V - v0));
    const float* gGl = reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K;
    for (int idx = tid; idx < D; idx += blockDim.x) sGl[idx] = idx < K ? gGl[idx] : 0.f;
    if (!a.prescan) {
      T* gdh = reinterpret_cast<T*>(a.ws + a.BL.dh) + ch * (size_t)K * V;
      for (int idx = tid; idx < K * kBV; idx += blockDim.x) {
        int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gdh[(size_t)r * V + col] = from_f<T>(sDH[r * LDB + cc]);
      }
    }
    __syncthreads();
    // dVN = Aqk^T dO + Kd dh   (64 x 32)
    {
      float acc[1][2][4];
      acc_zero(acc);
      warp_mma<1, 2, P>(acc, sAqk + m0, 1, LDC, sDO + n0, LDB, 1, kChunk);
      warp_mma<1, 2, P>(acc, sKd + m0 * LD, LD, 1, sDH + n0, LDB, 1, D);
      acc_foreach(acc, [&](int rr, int cc, float val) { sDVN[(m0 + rr) * LDB + n0 + cc] = val; });
    }
    __syncthreads();
    if (!a.prescan) {
      T* gdvn = reinterpret_cast<T*>(a.ws + a.BL.dvn) + ch * tileV;
      for (int idx = tid; idx < kChunk * kBV; idx += blockDim.x) {
        int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gdvn[(size_t)r * V + col] = from_f<T>(sDVN[r * LDB + cc]);
      }
    }
    // dh <- gl*dh + Qg^T dO - W^T dVN   (D x 32)
    {
      constexpr int RT = D / 16;
      float acc[(RT + 7) / 8][2][4][4];
      for (int t = 0; t < (RT + 7) / 8; ++t) {
        int mt = warp + 8 * t;
        if (mt < RT) {
          float p1[1][4][4], p2[1][4][4];
          acc_zero(p1);
          acc_zero(p2);
          warp_mma<1, 4, P>(p1, sQg + mt * 16, 1, LD, sDO, LDB, 1, kChunk);
          warp_mma<1, 4, P>(p2, sW + mt * 16, 1, LD, sDVN, LDB, 1, kChunk);
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              acc[t][0][j][e] = p1[0][j][e];
              acc[t][1][j][e] = p2[0][j][e];
            }
        }
      }
      __syncthreads();
      for (int t = 0; t < (RT + 7) / 8; ++t) {
        int mt = warp + 8 * t;
        if (mt < RT) {
          float part[1][4][4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) part[0][j][e] = acc[t][0][j][e] - acc[t][1][j][e];
          acc_foreach(part, [&](int rr, int cc, float val) {
            int r = mt * 16 + rr;
            sDH[r * LDB + cc] = sGl[r] * sDH[r * LDB + cc] + val;
          });
        }
      }
      __syncthreads();
    }
  }
  if (a.dh0) {
    for (int idx = tid; idx < K * kBV; idx += blockDim.x) {
      int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
      if (col < V) a.dh0[(((int64_t)n * H + h) * K + r) * V + col] = sDH[r * LDB + cc];
    }
  }
}

// ---------------------------------------------------------------------------

template <int D>
struct BIntraSmem {
  static constexpr int LD = D + 4;
  static constexpr int LDC = kChunk + 4;
  static constexpr int LDB = kBV + 4;
  static constexpr int phaseV = 2 * D * LDB + 6 * kChunk * LDB;
  static constexpr int colblk = 7 * kChunk * LDB + 32 * LDB;
  static constexpr int phaseK = 2 * kChunk * LDC + 3 * kChunk * LD + colblk;
  static constexpr int region = phaseV > phaseK ? phaseV : phaseK;
  static constexpr int misc = D + 4 * kChunk + 64;
  static constexpr int floats = kChunk * LDC + misc + region;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
  static_assert(2 * kChunk * LD <= region, "q/k staging must fit the work region");
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) k_bwd_intra(BwdIntraArgs a) {
  using S = BIntraSmem<D>;
  constexpr int LD = S::LD, LDC = S::LDC, LDB = S::LDB;
  constexpr int P = Passes<T>::value;
  constexpr int NT = D / 16;
  extern __shared__ __align__(16) float sm[];
  float* sA = sm;                        // [64][LDC]
  float* sDGL = sA + kChunk * LDC;       // [D] d(gl)
  float* sRq = sDGL + D;                 // [64] rsqrt norms of q rows
  float* sRk = sRq + kChunk;             // [64] ... of k rows
  float* sDiag = sRk + kChunk;           // [64] diagonal of dAqk
  float* sGLc = sDiag + kChunk;          // [32] d(G_last) of the current key block
  int* sFlag = reinterpret_cast<int*>(sGLc + 32);
  float* R = sm + kChunk * LDC + S::misc;
  // phase V
  float* sHs = R;
  float* sDHs = sHs + D * LDB;
  float* sDOs = sDHs + D * LDB;
  float* sVNs = sDOs + kChunk * LDB;
  float* sDVNs = sVNs + kChunk * LDB;
  float* sVs = sDVNs + kChunk * LDB;
  float* sWs = sVs + kChunk * LDB;
  float* sZs = sWs + kChunk * LDB;
  // phase K
  float* sDAqk = R;
  float* sDAkk = sDAqk + kChunk * LDC;
  float* sDQ = sDAkk + kChunk * LDC;     // [64][LD] dq (pre-norm)
  float* sDKn = sDQ + kChunk * LD;       // [64][LD] dKd -> Kd part of dk -> dk (pre-norm)
  float* sDKB = sDKn + kChunk * LD;      // [64][LD] dW -> d(b*k)
  float* sCq = sDKB + kChunk * LD;       // [64][LDB] key-block buffers
  float* sCk = sCq + kChunk * LDB;
  float* sCb = sCk + kChunk * LDB;
  float* sCg = sCb + kChunk * LDB;
  float* sCx = sCg + kChunk * LDB;       // scaled keys, then dG
  float* sCy = sCx + kChunk * LDB;       // Kd part of dG, shifted one row down
  float* sCd = sCy + kChunk * LDB;       // score i-side gradient of k
  float* sCl = sCd + kChunk * LDB;       // [32][LDB]
  float* sT = sCq;                       // [64][LDC] temp, aliases the key-block buffers

  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, K = a.K, V = a.V;
  const ChunkPos cp = chunk_pos(a.seqs, c);
  const int len = cp.len;
  const int64_t ldk = (int64_t)H * K, ldv = (int64_t)H * V;
  const int64_t offk = cp.row0 * ldk + (int64_t)h * K;
  const int64_t offv = cp.row0 * ldv + (int64_t)h * V;
  const size_t ch = (size_t)c * H + h;
  const T* gq = reinterpret_cast<const T*>(a.q) + offk;
  const T* gk = reinterpret_cast<const T*>(a.k) + offk;
  const T* gb = reinterpret_cast<const T*>(a.b) + offk;
  const float* gg = a.g + offk;

  // ---- phase 0: row norms of q and k (from staged tiles), A ----------------
  {
    float* tq = R;
    float* tk = R + kChunk * LD;
    load_tile<T, kChunk, D>(tq, LD, gq, ldk, len, K);
    load_tile<T, kChunk, D>(tk, LD, gk, ldk, len, K);
    load_tile<T, kChunk, kChunk>(sA, LDC,
                                 reinterpret_cast<const T*>(a.saved + a.L.a) + ch * kChunk * kChunk,
                                 kChunk, kChunk, kChunk);
    for (int idx = tid; idx < D; idx += blockDim.x) sDGL[idx] = 0.f;
    __syncthreads();
    for (int r = warp; r < kChunk; r += kThreads / 32) {
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int cc = lane; cc < D; cc += 32) {
        float x = tq[r * LD + cc], y = tk[r * LD + cc];
        sq += x * x;
        sk += y * y;
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      if (lane == 0) {
        sRq[r] = a.l2norm ? rsqrtf(sq + kNormEps) : 1.f;
        sRk[r] = a.l2norm ? rsqrtf(sk + kNormEps) : 1.f;
      }
    }
    __syncthreads();
  }

  // ---- phase V ------------------------------------------------------------
  const int wr = warp & 3, wc = warp >> 2, m0 = wr * 16;
  const int n0k = wc * (D / 2);
  float accQ[1][NT][4], accKd[1][NT][4], accW[1][NT][4], accAqk[1][4][4], accDA[1][4][4];
  acc_zero(accQ);
  acc_zero(accKd);
  acc_zero(accW);
  acc_zero(accAqk);
  acc_zero(accDA);
  const T* gh = reinterpret_cast<const T*>(a.saved + a.L.h) + ch * (size_t)K * V;
  const T* gdh = reinterpret_cast<const T*>(a.ws + a.BL.dh) + ch * (size_t)K * V;
  const T* gvn = reinterpret_cast<const T*>(a.saved + a.L.vn) + ch * (size_t)kChunk * V;
  const T* gdvn = reinterpret_cast<const T*>(a.ws + a.BL.dvn) + ch * (size_t)kChunk * V;
  const T* gdo = reinterpret_cast<const T*>(a.dout) + offv;
  const T* gv = reinterpret_cast<const T*>(a.v) + offv;
  const T* gw = reinterpret_cast<const T*>(a.w) + offv;
  T* gdv = reinterpret_cast<T*>(a.dv) + offv;
  T* gdw = reinterpret_cast<T*>(a.dw) + offv;
  for (int v0 = 0; v0 < V; v0 += kBV) {
    const int nv = min(kBV, V - v0);
    load_tile<T, D, kBV>(sHs, LDB, gh + v0, V, K, nv);
    load_tile<T, D, kBV>(sDHs, LDB, gdh + v0, V, K, nv);
    load_tile<T, kChunk, kBV>(sDOs, LDB, gdo + v0, ldv, len, nv);
    load_tile<T, kChunk, kBV>(sVNs, LDB, gvn + v0, V, kChunk, nv);
    load_tile<T, kChunk, kBV>(sDVNs, LDB, gdvn + v0, V, kChunk, nv);
    load_tile<T, kChunk, kBV>(sVs, LDB, gv + v0, ldv, len, nv);
    load_tile<T, kChunk, kBV>(sWs, LDB, gw + v0, ldv, len, nv);
    __syncthreads();
    for (int idx = tid; idx < kChunk * kBV; idx += blockDim.x) {
      int r = idx / kBV, cc = idx - r * kBV;
      sZs[r * LDB + cc] = sVs[r * LDB + cc] * sWs[r * LDB + cc];
    }
    if (tid < D) {
      float s = 0.f;
#pragma unroll 8
      for (int cc = 0; cc < kBV; ++cc) s += sHs[tid * LDB + cc] * sDHs[tid * LDB + cc];
      sDGL[tid] += s;
    }
    __syncthreads();
    warp_mma<1, NT, P>(accQ, sDOs + m0 * LDB, LDB, 1, sHs + n0k * LDB, 1, LDB, kBV);
    warp_mma<1, NT, P>(accKd, sVNs + m0 * LDB, LDB, 1, sDHs + n0k * LDB, 1, LDB, kBV);
    warp_mma<1, NT, P>(accW, sDVNs + m0 * LDB, LDB, 1, sHs + n0k * LDB, 1, LDB, kBV);
    warp_mma<1, 4, P>(accAqk, sDOs + m0 * LDB, LDB, 1, sVNs + (32 * wc) * LDB, 1, LDB, kBV);
    warp_mma<1, 4, P>(accDA, sDVNs + m0 * LDB, LDB, 1, sZs + (32 * wc) * LDB, 1, LDB, kBV);
    {
      float accZ[1][2][4];
      acc_zero(accZ);
      warp_mma<1, 2, P>(accZ, sA + m0, 1, LDC, sDVNs + 16 * wc, LDB, 1, kChunk);
      acc_foreach(accZ, [&](int rr, int cc, float val) {
        int r = m0 + rr, col = 16 * wc + cc;
        if (r < len && col < nv) {
          gdv[r * ldv + v0 + col] = from_f<T>(val * sWs[r * LDB + col]);
          gdw[r * ldv + v0 + col] = from_f<T>(val * sVs[r * LDB + col]);
        }
      });
    }
    __syncthreads();
  }

  // ---- dump value-side results into the key-side buffers -------------------
  // The diagonal of dAqk (a token's score with itself) is kept apart: its
  // contributions to dG through q and through k cancel exactly, so it is
  // added to dq and dk only after dG is formed (no rounding residue in dg).
  acc_foreach(accQ, [&](int rr, int cc, float val) { sDQ[(m0 + rr) * LD + n0k + cc] = val; });
  acc_foreach(accKd, [&](int rr, int cc, float val) { sDKn[(m0 + rr) * LD + n0k + cc] = val; });
  acc_foreach(accW, [&](int rr, int cc, float val) { sDKB[(m0 + rr) * LD + n0k + cc] = -val; });
  acc_foreach(accAqk, [&](int rr, int cc, float val) {
    int r = m0 + rr, i = 32 * wc + cc;
    sDAqk[r * LDC + i] = (i < r) ? val : 0.f;
    if (i == r) sDiag[r] = val;
  });
  __syncthreads();

  // ---- key blocks, pass 1: dA += dW E^T ------------------------------------
  auto load_cols = [&](int c0, bool need_q) {
    const int nk = min(32, K - c0);
    if (need_q) load_tile<T, kChunk, 32>(sCq, LDB, gq + c0, ldk, len, nk);
    load_tile<T, kChunk, 32>(sCk, LDB, gk + c0, ldk, len, nk);
    load_tile<T, kChunk, 32>(sCb, LDB, gb + c0, ldk, len, nk);
    load_tile<float, kChunk, 32>(sCg, LDB, gg + c0, ldk, len, nk);
    __syncthreads();
    for (int idx = tid; idx < kChunk * 32; idx += blockDim.x) {
      int r = idx >> 5, cc = idx & 31;
      sCk[r * LDB + cc] *= sRk[r];
      if (need_q) sCq[r * LDB + cc] *= sRq[r];
    }
    col_cumsum64<32>(sCg, LDB, kLog2e, sCl);
  };
  for (int c0 = 0; c0 < K; c0 += 32) {
    load_cols(c0, false);
    for (int idx = tid; idx < kChunk * 32; idx += blockDim.x) {
      int r = idx >> 5, cc = idx & 31;
      sCx[r * LDB + cc] = sCb[r * LDB + cc] * sCk[r * LDB + cc] * exp2f(sCg[r * LDB + cc]);
    }
    __syncthreads();
    warp_mma<1, 4, P>(accDA, sDKB + m0 * LD + c0, LD, 1, sCx + (32 * wc) * LDB, 1, LDB, 32);
    __syncthreads();
  }
  // dAkk = -tril_strict(A^T dA A^T)
  acc_foreach(accDA, [&](int rr, int cc, float val) { sT[(m0 + rr) * LDC + 32 * wc + cc] = val; });
  __syncthreads();
  {
    float t1[1][4][4];
    acc_zero(t1);
    warp_mma<1, 4, P>(t1, sA + m0, 1, LDC, sT + 32 * wc, LDC, 1, kChunk);
    __syncthreads();
    acc_foreach(t1, [&](int rr, int cc, float val) { sT[(m0 + rr) * LDC + 32 * wc + cc] = val; });
    __syncthreads();
    acc_zero(t1);
    warp_mma<1, 4, P>(t1, sT + m0 * LDC, LDC, 1, sA + (32 * wc) * LDC, 1, LDC, kChunk);
    acc_foreach(t1, [&](int rr, int cc, float val) {
      int r = m0 + rr, i = 32 * wc + cc;
      sDAkk[r * LDC + i] = (i < r) ? -val : 0.f;
    });
    __syncthreads();
  }

  // ---- key blocks, pass 2 -------------------------------------------------
  T* gdq = reinterpret_cast<T*>(a.dq) + offk;
  T* gdk = reinterpret_cast<T*>(a.dk) + offk;
  T* gdb = reinterpret_cast<T*>(a.db) + offk;
  float* gdg = a.dg + offk;
  const float* gGl = reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K;
  const float scale = a.scale;
  for (int c0 = 0; c0 < K; c0 += 32) {
    const int nk = min(32, K - c0);
    load_cols(c0, true);
    if (tid == 0) sFlag[0] = 1;
    __syncthreads();
    for (int idx = tid; idx < 4 * 32; idx += blockDim.x) {
      int bI = idx >> 5, cc = idx & 31;
      float rng = sCg[(16 * bI) * LDB + cc] - sCg[(16 * bI + 15) * LDB + cc];
      if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
    }
    // dE = A^T dW for this block (64 x 32): warp tile 16 x 16
    float accE[1][2][4];
    acc_zero(accE);
    warp_mma<1, 2, P>(accE, sA + m0, 1, LDC, sDKB + c0 + 16 * wc, LD, 1, kChunk);
    __syncthreads();
    const bool safe = sFlag[0] != 0;
    acc_foreach(accE, [&](int rr, int cc, float val) {
      int r = m0 + rr, col = 16 * wc + cc;
      sDKB[r * LD + c0 + col] = val * exp2f(sCg[r * LDB + col]);
    });
    // dq <- scale 2^G dQg;  Kd part of dk <- dKd 2^(G_L - G);  its dG share
    // X_r = k_r * (Kd part)_r goes to sCy shifted one row down, so that a
    // prefix scan yields sum_{r<t} X_r without subtracting anything.
    for (int idx = tid; idx < kChunk * 32; idx += blockDim.x) {
      int r = idx >> 5, cc = idx & 31;
      float G = sCg[r * LDB + cc], GL = sCg[(kChunk - 1) * LDB + cc];
      sDQ[r * LD + c0 + cc] *= scale * exp2f(G);
      float kd = sDKn[r * LD + c0 + cc] * exp2f(GL - G);
      sDKn[r * LD + c0 + cc] = kd;
      if (r + 1 < kChunk) sCy[(r + 1) * LDB + cc] = sCk[r * LDB + cc] * kd;
      if (r == 0) sCy[cc] = 0.f;
      sCd[r * LDB + cc] = 0.f;
    }
    if (tid < 32) {
      float gl = (tid < nk) ? gGl[c0 + tid] : 0.f;
      sGLc[tid] = sDGL[c0 + tid] * gl;
    }
    // score blocks
    for (int bI = 0; bI < 4; ++bI) {
      const int r0 = 16 * bI, ni = 16 * (bI + 1);
      const int jmax = safe ? ni : 16 * bI;
      __syncthreads();
      for (int idx = tid; idx < 16 * 32; idx += blockDim.x) {
        int rr = idx >> 5, cc = idx & 31, r = r0 + rr;
        float f = exp2f(sCg[r * LDB + cc] - sCg[r0 * LDB + cc]);
        sCl[rr * LDB + cc] = scale * sCq[r * LDB + cc] * f;
        sCl[(16 + rr) * LDB + cc] = sCb[r * LDB + cc] * sCk[r * LDB + cc] * f;
      }
      for (int idx = tid; idx < ni * 32; idx += blockDim.x) {
        int i = idx >> 5, cc = idx & 31;
        float e = fminf(sCg[r0 * LDB + cc] - sCg[i * LDB + cc], 120.f);
        sCx[i * LDB + cc] = sCk[i * LDB + cc] * exp2f(e);
      }
      __syncthreads();
      if (jmax > 0) {
        // X = [dAqk_I ; dAkk_I] Ks : 8 items of 16 x 8
        {
          const int which = warp >> 2, nt = warp & 3;
          float acc[1][1][4];
          acc_zero(acc);
          warp_mma<1, 1, P>(acc, (which ? sDAkk : sDAqk) + r0 * LDC, LDC, 1, sCx + 8 * nt, LDB, 1,
                            jmax);
          acc_foreach(acc, [&](int rr, int cc, float val) {
            int r = r0 + rr, col = 8 * nt + cc;
            float f = exp2f(sCg[r * LDB + col] - sCg[r0 * LDB + col]);
            if (which == 0)
              sDQ[r * LD + c0 + col] += scale * val * f;
            else
              sDKB[r * LD + c0 + col] += val * f;
          });
        }
        // Y = dAqk_I^T (scale Qs) + dAkk_I^T KBs : (jmax x 32), items of 16 x 8
        const int nitems = (jmax / 16) * 4;
        for (int it = warp; it < nitems; it += kThreads / 32) {
          const int mt = it >> 2, nt = it & 3;
          float acc[1][1][4];
          acc_zero(acc);
          warp_mma<1, 1, P>(acc, sDAqk + r0 * LDC + 16 * mt, 1, LDC, sCl + 8 * nt, LDB, 1, 16);
          warp_mma<1, 1, P>(acc, sDAkk + r0 * LDC + 16 * mt, 1, LDC, sCl + 16 * LDB + 8 * nt, LDB,
                            1, 16);
          acc_foreach(acc, [&](int rr, int cc, float val) {
            int i = 16 * mt + rr, col = 8 * nt + cc;
            float e = fminf(sCg[r0 * LDB + col] - sCg[i * LDB + col], 120.f);
            sCd[i * LDB + col] += val * exp2f(e);
          });
        }
      }
      if (!safe) {
        __syncthreads();
        // exact diagonal block (off-diagonal pairs only; the diagonal itself
        // is handled apart, see above)
        for (int idx = tid; idx < 16 * 32; idx += blockDim.x) {
          int rr = idx >> 5, cc = idx & 31, r = r0 + rr;
          float sq = 0.f, sk = 0.f, sy = 0.f;
          for (int ii = 0; ii < rr; ++ii) {
            int i = r0 + ii;
            float e = exp2f(sCg[r * LDB + cc] - sCg[i * LDB + cc]) * sCk[i * LDB + cc];
            sq += sDAqk[r * LDC + i] * e;
            sk += sDAkk[r * LDC + i] * e;
          }
          for (int r2 = rr + 1; r2 < 16; ++r2) {
            int rb = r0 + r2;
            float e = exp2f(sCg[rb * LDB + cc] - sCg[r * LDB + cc]);
            float t = scale * sDAqk[rb * LDC + r] * sCq[rb * LDB + cc] +
                      sDAkk[rb * LDC + r] * sCb[rb * LDB + cc] * sCk[rb * LDB + cc];
            sy += t * e;
          }
          sDQ[r * LD + c0 + cc] += scale * sq;
          sDKB[r * LD + c0 + cc] += sk;
          sCd[r * LDB + cc] += sy;
        }
      }
    }
    __syncthreads();
    // per-element chain: dG (without the Kd part and the diagonal), db, dk
    for (int idx = tid; idx < kChunk * 32; idx += blockDim.x) {
      int r = idx >> 5, cc = idx & 31;
      float qn = sCq[r * LDB + cc], kn = sCk[r * LDB + cc], bb = sCb[r * LDB + cc];
      float dqn = sDQ[r * LD + c0 + cc], dkb = sDKB[r * LD + c0 + cc], dy = sCd[r * LDB + cc];
      float dG = qn * dqn + bb * kn * dkb - kn * dy;
      if (r == len - 1) dG += sGLc[cc];
      sCx[r * LDB + cc] = dG;
      const float dgn = scale * sDiag[r];
      sDQ[r * LD + c0 + cc] = dqn + dgn * kn;
      sDKn[r * LD + c0 + cc] += dy + dkb * bb + dgn * qn;
      if (r < len && cc < nk) gdb[(int64_t)r * ldk + c0 + cc] = from_f<T>(dkb * kn);
    }
    __syncthreads();
    // dg_t = sum_{r>=t} dG_r + sum_{r<t} X_r
    col_scan64<32, true>(sCx, LDB, sCl);
    col_scan64<32, false>(sCy, LDB, sCl);
    for (int idx = tid; idx < kChunk * 32; idx += blockDim.x) {
      int r = idx >> 5, cc = idx & 31;
      if (r < len && cc < nk)
        gdg[(int64_t)r * ldk + c0 + cc] = sCx[r * LDB + cc] + sCy[r * LDB + cc];
    }
    __syncthreads();
  }

  // ---- l2norm backward and dq / dk out -------------------------------------
  {
    // stage the raw q, k rows in the key-block area (free now; it does not
    // overlap sDQ / sDKn)
    static_assert(2 * kChunk * LD <= S::colblk, "q/k staging must fit the key-block area");
    float* tq = sCq;
    float* tk = sCq + kChunk * LD;
    load_tile<T, kChunk, D>(tq, LD, gq, ldk, len, K);
    load_tile<T, kChunk, D>(tk, LD, gk, ldk, len, K);
    __syncthreads();
    for (int r = warp; r < len; r += kThreads / 32) {
      const float rq = sRq[r], rk = sRk[r];
      float pq = 0.f, pk = 0.f;
      if (a.l2norm) {
        for (int cc = lane; cc < K; cc += 32) {
          pq += tq[r * LD + cc] * rq * sDQ[r * LD + cc];
          pk += tk[r * LD + cc] * rk * sDKn[r * LD + cc];
        }
        pq = warp_sum(pq);
        pk = warp_sum(pk);
      }
      for (int cc = lane; cc < K; cc += 32) {
        float dqv = sDQ[r * LD + cc], dkv = sDKn[r * LD + cc];
        if (a.l2norm) {
          dqv = (dqv - tq[r * LD + cc] * rq * pq) * rq;
          dkv = (dkv - tk[r * LD + cc] * rk * pk) * rk;
        }
        gdq[r * ldk + cc] = from_f<T>(dqv);
        gdk[r * ldk + cc] = from_f<T>(dkv);
      }
    }
  }
}

// ---------------------------------------------------------------------------
template <typename T, int D>
cudaError_t launch_bwd_state(const BwdStateArgs& a, cudaStream_t st) {
  auto kern = k_bwd_state<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)BStateSmem<D>::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid((a.V + kBV - 1) / kBV, a.seqs.n_seqs * a.H);
  kern<<<grid, kThreads, BStateSmem<D>::bytes, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_bwd_intra(const BwdIntraArgs& a, cudaStream_t st) {
  auto kern = k_bwd_intra<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)BIntraSmem<D>::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(a.seqs.n_chunks, a.H);
  kern<<<grid, kThreads, BIntraSmem<D>::bytes, st>>>(a);
  return cudaGetLastError();
}

#define GDN2_INST_BWD(T, D)                                                           \
  template cudaError_t launch_bwd_state<T, D>(const BwdStateArgs&, cudaStream_t);    \
  template cudaError_t launch_bwd_intra<T, D>(const BwdIntraArgs&, cudaStream_t);
GDN2_INST_BWD(float, 64)
GDN2_INST_BWD(float, 128)
GDN2_INST_BWD(__nv_bfloat16, 64)
GDN2_INST_BWD(__nv_bfloat16, 128)
GDN2_INST_BWD(__half, 64)
GDN2_INST_BWD(__half, 128)

}  // namespace gdn2
