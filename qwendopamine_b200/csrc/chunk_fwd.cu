// chunk_fwd.cu -- chunkwise GDN-2 forward on B200.
//
// Phase 1, k_fwd_intra: one CTA per (chunk, head), fully parallel.  Replaces
//   the Triton kernels K1/K3/K4 and FLA's chunk_local_cumsum / l2norm_fwd
//   (chunk_gdn2.py:175-1162).  For one chunk of 64 tokens it computes the
//   chunk-local cumulative log2 decay G, the causal score matrices
//     Aqk[r,i] = scale * sum_c q[r,c] k[i,c] 2^(G[r,c]-G[i,c])   (i <= r)
//     Akk[r,i] =         sum_c (b*k)[r,c] k[i,c] 2^(G[r,c]-G[i,c]) (i < r)
//   the unit-lower inverse A = (I + Akk)^-1, and the WY factors
//     W = A (b*k*2^G),  U = A (w*v),  Qg = scale*q*2^G,  Kd = k*2^(G_last-G).
//   Decays are always relative: the score blocks use per-16-row reference
//   rows (as the Triton path does, chunk_gdn2.py:584-589), never 1/gamma.
//
// Phase 2, k_fwd_state: one CTA per (sequence, head, 32-column value tile),
//   sequential over the sequence's chunks.  Replaces K6 + K7
//   (chunk_kda.py:1302-1730 and FLA chunk_gla_fwd_o_gk): the fp32 state tile
//   stays in shared memory and each step does
//     VN = U - W h;  o = Qg h + Aqk VN;  h <- 2^G_last * h + Kd^T VN.
//   The same kernel, in pre-scan mode, carries [h_e | M] (K x (V+K)) from
//   [0 | I] with no output, which is the context-parallel span map.
#include "chunk_args.cuh"
#include "inverse.cuh"

namespace gdn2 {

template <int D>
struct IntraSmem {
  static constexpr int LD = D + 4;     // row stride of 64 x D tiles
  static constexpr int LDC = kChunk + 4;  // row stride of 64 x 64 tiles
  static constexpr int floats = 5 * kChunk * LD + 32 * LD + 2 * kChunk * LDC + D + 32;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) k_fwd_intra(FwdIntraArgs a) {
  using S = IntraSmem<D>;
  constexpr int LD = S::LD, LDC = S::LDC;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sG = sm;                  // [64][LD] log2-domain chunk cumsum of g
  float* sQ = sG + kChunk * LD;    // normalised q
  float* sK = sQ + kChunk * LD;    // normalised k
  float* sKB = sK + kChunk * LD;   // b*k, later b*k*2^G
  float* sX = sKB + kChunk * LD;   // scratch: reference-scaled keys
  float* sL = sX + kChunk * LD;    // [32][LD] scratch: [Qs; KBs]
  float* sAqk = sL + 32 * LD;      // [64][LDC]
  float* sAkk = sAqk + kChunk * LDC;
  float* sMisc = sAkk + kChunk * LDC;  // [D] + flags
  int* sFlag = reinterpret_cast<int*>(sMisc + D);

  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, K = a.K, V = a.V;
  const ChunkPos cp = chunk_pos(a.seqs, c);
  const int len = cp.len;
  const int64_t ldk = (int64_t)H * K, ldv = (int64_t)H * V;
  const int64_t offk = cp.row0 * ldk + (int64_t)h * K;
  const int64_t offv = cp.row0 * ldv + (int64_t)h * V;

  // ---- loads ---------------------------------------------------------------
  load_tile<float, kChunk, D>(sG, LD, a.g + offk, ldk, len, K);
  load_tile<T, kChunk, D>(sQ, LD, reinterpret_cast<const T*>(a.q) + offk, ldk, len, K);
  load_tile<T, kChunk, D>(sK, LD, reinterpret_cast<const T*>(a.k) + offk, ldk, len, K);
  load_tile<T, kChunk, D>(sKB, LD, reinterpret_cast<const T*>(a.b) + offk, ldk, len, K);
  for (int idx = tid; idx < kChunk * LDC; idx += blockDim.x) {
    sAqk[idx] = 0.f;
    sAkk[idx] = 0.f;
  }
  if (tid == 0) sFlag[0] = 1;
  __syncthreads();

  // chunk-local cumulative decay (log2 domain)
  col_cumsum64<D>(sG, LD, kLog2e, sX);
  // L2 normalisation of q and k rows: x * rsqrt(sum x^2 + eps)
  if (a.l2norm) {
    for (int r = warp; r < kChunk; r += kThreads / 32) {
      float sq = 0.f, sk = 0.f;
      for (int cc = lane; cc < D; cc += 32) {
        float x = sQ[r * LD + cc], y = sK[r * LD + cc];
        sq += x * x;
        sk += y * y;
      }
      sq = rsqrtf(warp_sum(sq) + kNormEps);
      sk = rsqrtf(warp_sum(sk) + kNormEps);
      for (int cc = lane; cc < D; cc += 32) {
        sQ[r * LD + cc] *= sq;
        sK[r * LD + cc] *= sk;
      }
    }
  }
  __syncthreads();
  for (int idx = tid; idx < kChunk * D; idx += blockDim.x) {
    int r = idx / D, cc = idx - r * D;
    sKB[r * LD + cc] *= sK[r * LD + cc];
  }
  // diagonal-block safety: the largest within-block decay range
  for (int idx = tid; idx < 4 * D; idx += blockDim.x) {
    int bI = idx / D, cc = idx - bI * D;
    float rng = sG[(16 * bI) * LD + cc] - sG[(16 * bI + 15) * LD + cc];
    if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
  }
  __syncthreads();
  const bool safe = sFlag[0] != 0;

  // ---- score blocks, one 16-row block-row at a time ------------------------
  for (int bI = 0; bI < 4; ++bI) {
    const int r0 = 16 * bI, ni = 16 * (bI + 1);
    for (int idx = tid; idx < 16 * D; idx += blockDim.x) {
      int rr = idx / D, cc = idx - rr * D;
      float f = exp2f(sG[(r0 + rr) * LD + cc] - sG[r0 * LD + cc]);
      sL[rr * LD + cc] = sQ[(r0 + rr) * LD + cc] * f;
      sL[(16 + rr) * LD + cc] = sKB[(r0 + rr) * LD + cc] * f;
    }
    for (int idx = tid; idx < ni * D; idx += blockDim.x) {
      int i = idx / D, cc = idx - i * D;
      float e = fminf(sG[r0 * LD + cc] - sG[i * LD + cc], 120.f);
      sX[i * LD + cc] = sK[i * LD + cc] * exp2f(e);
    }
    __syncthreads();
    // [32 x ni] = sL[32 x D] * sX[ni x D]^T ; items of 16x16, 2*(bI+1) of them
    const int nitems = 2 * (bI + 1);
    for (int it = warp; it < nitems; it += kThreads / 32) {
      const int mt = it & 1, nt = it >> 1;
      float acc[1][2][4];
      acc_zero(acc);
      warp_mma<1, 2, P>(acc, sL + mt * 16 * LD, LD, 1, sX + nt * 16 * LD, 1, LD, D);
      acc_foreach(acc, [&](int rr, int cc, float val) {
        int col = nt * 16 + cc;
        if (mt == 0) {
          int row = r0 + rr;
          if (col <= row) sAqk[row * LDC + col] = a.scale * val;
        } else {
          int row = r0 + rr;
          if (col < row) sAkk[row * LDC + col] = val;
        }
      });
    }
    __syncthreads();
  }
  if (!safe) {
    // exact diagonal blocks: 2^(G_r - G_i) per element, no factoring
    for (int idx = tid; idx < 4 * 256; idx += blockDim.x) {
      int bI = idx >> 8, e = idx & 255, rr = e >> 4, ii = e & 15;
      if (ii > rr) continue;
      int r = 16 * bI + rr, i = 16 * bI + ii;
      float sq = 0.f, skk = 0.f;
      for (int cc = 0; cc < D; ++cc) {
        float f = exp2f(sG[r * LD + cc] - sG[i * LD + cc]) * sK[i * LD + cc];
        sq += sQ[r * LD + cc] * f;
        skk += sKB[r * LD + cc] * f;
      }
      sAqk[r * LDC + i] = a.scale * sq;
      if (ii < rr) sAkk[r * LDC + i] = skk;
    }
    __syncthreads();
  }

  // ---- Qg, Kd, gl, Aqk out ----------------------------------------------
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const size_t ch = (size_t)c * H + h;
  T* gQg = reinterpret_cast<T*>(a.saved + a.L.qg) + ch * tileK;
  T* gKd = reinterpret_cast<T*>(a.saved + a.L.kd) + ch * tileK;
  T* gW = reinterpret_cast<T*>(a.saved + a.L.w) + ch * tileK;
  T* gU = reinterpret_cast<T*>(a.saved + a.L.u) + ch * tileV;
  T* gAqk = reinterpret_cast<T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk;
  T* gA = reinterpret_cast<T*>(a.saved + a.L.a) + ch * kChunk * kChunk;
  float* gGl = reinterpret_cast<float*>(a.saved + a.L.gl) + ch * K;
  for (int idx = tid; idx < kChunk * K; idx += blockDim.x) {
    int r = idx / K, cc = idx - r * K;
    float G = sG[r * LD + cc], GL = sG[(kChunk - 1) * LD + cc];
    gQg[idx] = from_f<T>(a.scale * sQ[r * LD + cc] * exp2f(G));
    gKd[idx] = from_f<T>(sK[r * LD + cc] * exp2f(GL - G));
  }
  for (int idx = tid; idx < K; idx += blockDim.x) gGl[idx] = exp2f(sG[(kChunk - 1) * LD + idx]);
  for (int idx = tid; idx < kChunk * kChunk; idx += blockDim.x)
    gAqk[idx] = from_f<T>(sAqk[(idx >> 6) * LDC + (idx & 63)]);
  __syncthreads();

  // ---- A = (I + Akk)^-1 into sAqk's buffer --------------------------------
  float* sA = sAqk;
  unit_lower_inverse<LDC>(sAkk, sA, sX);
  for (int idx = tid; idx < kChunk * kChunk; idx += blockDim.x)
    gA[idx] = from_f<T>(sA[(idx >> 6) * LDC + (idx & 63)]);
  // E = b*k*2^G (in place), Z = w*v into sQ (sQ, sK are free now)
  for (int idx = tid; idx < kChunk * D; idx += blockDim.x) {
    int r = idx / D, cc = idx - r * D;
    sKB[r * LD + cc] *= exp2f(sG[r * LD + cc]);
  }
  load_tile<T, kChunk, D>(sQ, LD, reinterpret_cast<const T*>(a.v) + offv, ldv, len, V);
  load_tile<T, kChunk, D>(sK, LD, reinterpret_cast<const T*>(a.w) + offv, ldv, len, V);
  __syncthreads();
  for (int idx = tid; idx < kChunk * D; idx += blockDim.x) {
    int r = idx / D, cc = idx - r * D;
    sQ[r * LD + cc] *= sK[r * LD + cc];
  }
  __syncthreads();

  // W = A E, U = A Z : warp tile 16 x D/2
  {
    constexpr int NT = D / 16;
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * (D / 2);
    float acc[1][NT][4];
    acc_zero(acc);
    warp_mma<1, NT, P>(acc, sA + m0 * LDC, LDC, 1, sKB + n0, LD, 1, kChunk);
    acc_foreach(acc, [&](int rr, int cc, float val) {
      int r = m0 + rr, col = n0 + cc;
      if (col < K) gW[r * K + col] = from_f<T>(val);
    });
    acc_zero(acc);
    warp_mma<1, NT, P>(acc, sA + m0 * LDC, LDC, 1, sQ + n0, LD, 1, kChunk);
    acc_foreach(acc, [&](int rr, int cc, float val) {
      int r = m0 + rr, col = n0 + cc;
      if (col < V) gU[r * V + col] = from_f<T>(val);
    });
  }
}

// ---------------------------------------------------------------------------
// state pass
// ---------------------------------------------------------------------------

template <int D>
struct StateSmem {
  static constexpr int LD = D + 4;
  static constexpr int LDC = kChunk + 4;
  static constexpr int LDB = kBV + 4;
  static constexpr int floats = 3 * kChunk * LD + kChunk * LDC + 2 * kChunk * LDB + D * LDB + D;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) k_fwd_state(FwdStateArgs a) {
  using S = StateSmem<D>;
  constexpr int LD = S::LD, LDC = S::LDC, LDB = S::LDB;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sQg = sm;
  float* sKd = sQg + kChunk * LD;
  float* sW = sKd + kChunk * LD;
  float* sAqk = sW + kChunk * LD;
  float* sU = sAqk + kChunk * LDC;   // [64][LDB]
  float* sVN = sU + kChunk * LDB;    // [64][LDB]
  float* sH = sVN + kChunk * LDB;    // [D][LDB]
  float* sGl = sH + D * LDB;         // [D]

  const int tid = threadIdx.x, warp = tid >> 5;
  const int H = a.H, K = a.K, V = a.V;
  const int nh = blockIdx.y, n = nh / H, h = nh - n * H;
  const int v0 = blockIdx.x * kBV;
  const int Vx = a.prescan ? V + K : V;  // carried columns
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];

  // initial state tile
  for (int idx = tid; idx < D * kBV; idx += blockDim.x) {
    int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
    float x = 0.f;
    if (r < K && col < Vx) {
      if (a.prescan) {
        x = (col >= V && col - V == r) ? 1.f : 0.f;
      } else if (a.h0) {
        x = a.h0[(((int64_t)n * H + h) * K + r) * V + col];
      }
    }
    sH[r * LDB + cc] = x;
  }

  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const int64_t ldo = (int64_t)H * V;
  for (int c = c_begin; c < c_end; ++c) {
    const size_t ch = (size_t)c * H + h;
    const T* gQg = reinterpret_cast<const T*>(a.saved + a.L.qg) + ch * tileK;
    const T* gKd = reinterpret_cast<const T*>(a.saved + a.L.kd) + ch * tileK;
    const T* gW = reinterpret_cast<const T*>(a.saved + a.L.w) + ch * tileK;
    const T* gU = reinterpret_cast<const T*>(a.saved + a.L.u) + ch * tileV;
    const T* gAqk = reinterpret_cast<const T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk;
    const float* gGl = reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K;
    if (!a.prescan) load_tile<T, kChunk, D>(sQg, LD, gQg, K, kChunk, K);
    load_tile<T, kChunk, D>(sKd, LD, gKd, K, kChunk, K);
    load_tile<T, kChunk, D>(sW, LD, gW, K, kChunk, K);
    if (!a.prescan) load_tile<T, kChunk, kChunk>(sAqk, LDC, gAqk, kChunk, kChunk, kChunk);
    // U tile (columns beyond V are the M part of the pre-scan: zero)
    load_tile<T, kChunk, kBV>(sU, LDB, gU + v0, V, kChunk, max(0, min(kBV, V - v0)));
    for (int idx = tid; idx < D; idx += blockDim.x) sGl[idx] = idx < K ? gGl[idx] : 0.f;
    if (!a.prescan) {
      // checkpoint of the state entering this chunk (for the backward)
      T* gh = reinterpret_cast<T*>(a.saved + a.L.h) + ch * (size_t)K * V;
      for (int idx = tid; idx < K * kBV; idx += blockDim.x) {
        int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gh[(size_t)r * V + col] = from_f<T>(sH[r * LDB + cc]);
      }
    }
    __syncthreads();

    // VN = U - W h  (64 x 32): warp tile 16 x 16
    const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 16;
    {
      float acc[1][2][4];
      acc_zero(acc);
      warp_mma<1, 2, P>(acc, sW + m0 * LD, LD, 1, sH + n0, LDB, 1, D);
      acc_foreach(acc, [&](int rr, int cc, float val) {
        int r = m0 + rr, col = n0 + cc;
        sVN[r * LDB + col] = sU[r * LDB + col] - val;
      });
    }
    __syncthreads();
    if (!a.prescan) {
      T* gVN = reinterpret_cast<T*>(a.saved + a.L.vn) + ch * tileV;
      for (int idx = tid; idx < kChunk * kBV; idx += blockDim.x) {
        int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gVN[(size_t)r * V + col] = from_f<T>(sVN[r * LDB + cc]);
      }
      // o = Qg h + Aqk VN
      const ChunkPos cp = chunk_pos(a.seqs, c);
      float acc[1][2][4];
      acc_zero(acc);
      warp_mma<1, 2, P>(acc, sQg + m0 * LD, LD, 1, sH + n0, LDB, 1, D);
      warp_mma<1, 2, P>(acc, sAqk + m0 * LDC, LDC, 1, sVN + n0, LDB, 1, kChunk);
      T* go = reinterpret_cast<T*>(a.o) + cp.row0 * ldo + (int64_t)h * V;
      acc_foreach(acc, [&](int rr, int cc, float val) {
        int r = m0 + rr, col = v0 + n0 + cc;
        if (r < cp.len && col < V) go[r * ldo + col] = from_f<T>(val);
      });
    }
    // h <- gl * h + Kd^T VN   (D x 32): warp tile 16 x 32, D/16 row tiles
    {
      constexpr int RT = D / 16;
      float acc[(RT + 7) / 8][4][4];
      acc_zero(acc);
      for (int t = 0; t < (RT + 7) / 8; ++t) {
        int mt = warp + 8 * t;
        if (mt < RT) {
          float part[1][4][4];
          acc_zero(part);
          warp_mma<1, 4, P>(part, sKd + mt * 16, 1, LD, sVN, LDB, 1, kChunk);
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[t][j][e] = part[0][j][e];
        }
      }
      __syncthreads();  // every read of sH, sKd, sVN is done
      for (int t = 0; t < (RT + 7) / 8; ++t) {
        int mt = warp + 8 * t;
        if (mt < RT) {
          float part[1][4][4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) part[0][j][e] = acc[t][j][e];
          acc_foreach(part, [&](int rr, int cc, float val) {
            int r = mt * 16 + rr;
            sH[r * LDB + cc] = sGl[r] * sH[r * LDB + cc] + val;
          });
        }
      }
      __syncthreads();
    }
  }

  // final state
  if (a.prescan) {
    for (int idx = tid; idx < K * kBV; idx += blockDim.x) {
      int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
      if (col < Vx) a.hm[(((int64_t)n * H + h) * K + r) * Vx + col] = sH[r * LDB + cc];
    }
  } else if (a.ht) {
    for (int idx = tid; idx < K * kBV; idx += blockDim.x) {
      int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
      if (col < V) a.ht[(((int64_t)n * H + h) * K + r) * V + col] = sH[r * LDB + cc];
    }
  }
}

// ---------------------------------------------------------------------------
// launchers
// ---------------------------------------------------------------------------
template <typename T, int D>
cudaError_t launch_fwd_intra(const FwdIntraArgs& a, cudaStream_t st) {
  auto kern = k_fwd_intra<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)IntraSmem<D>::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(a.seqs.n_chunks, a.H);
  kern<<<grid, kThreads, IntraSmem<D>::bytes, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_fwd_state(const FwdStateArgs& a, cudaStream_t st) {
  auto kern = k_fwd_state<T, D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)StateSmem<D>::bytes);
  if (e != cudaSuccess) return e;
  const int cols = a.prescan ? a.V + a.K : a.V;
  dim3 grid((cols + kBV - 1) / kBV, a.seqs.n_seqs * a.H);
  kern<<<grid, kThreads, StateSmem<D>::bytes, st>>>(a);
  return cudaGetLastError();
}

#define GDN2_INST_FWD(T, D)                                                            \
  template cudaError_t launch_fwd_intra<T, D>(const FwdIntraArgs&, cudaStream_t);     \
  template cudaError_t launch_fwd_state<T, D>(const FwdStateArgs&, cudaStream_t);
GDN2_INST_FWD(float, 64)
GDN2_INST_FWD(float, 128)
GDN2_INST_FWD(__nv_bfloat16, 64)
GDN2_INST_FWD(__nv_bfloat16, 128)
GDN2_INST_FWD(__half, 64)
GDN2_INST_FWD(__half, 128)

}  // namespace gdn2
