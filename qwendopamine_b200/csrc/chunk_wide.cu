// chunk_wide.cu -- chunkwise GDN-2 for head sizes above 128 (K, V <= 256).
//
// The reference accepts key heads up to 256 (chunk_gdn2.py:1380-1382) and
// value heads of expand_v * head_dim (gdn2.py:568-571).  The per-chunk tiles
// of such heads do not fit the shared memory of the kernels in chunk_fwd.cu /
// chunk_bwd.cu, so these kernels walk the key and value channels in 64-wide
// slabs (32-wide value tiles in the state passes).  Same mathematics and
// rounding points as the generic kernels, fp32 staging, tensor-core products
// on mma.sync TF32 (the 3-term split for fp32 inputs):
//
//  k_fwd_intra_wide (chunk, head): row norms over all K channels; per key
//      slab the chunk-local decay scan, the off-diagonal score blocks through
//      each block's first row (factors <= 1) and the diagonal blocks
//      elementwise (exact), accumulated over slabs; Qg, Kd, gl per slab;
//      A = (I + Akk)^-1; W = A E per key slab; U = A (w v) per value slab.
//  k_fwd_state_wide (sequence, head, 32 value columns): the K x 32 fp32 state
//      tile in shared memory; VN = U - W h and Qg h accumulated over key
//      slabs; o = Qg h + Aqk VN; h <- gl h + Kd^T VN per key slab.  Also the
//      context-parallel pre-scan ([h | M] over V + K columns from [0 | I]).
//  k_bwd_state_wide (sequence, head, 32 value columns), reverse: dVN =
//      Aqk^T dO + Kd dh over key slabs; dh <- gl dh + Qg^T dO - W^T dVN per
//      key slab.  Also the backward pre-scan.
//  k_bwd_intra_wide (chunk, head): a first pass over key slabs forms dA =
//      dVN (w v)^T + dW E^T together with dAqk, dv and dw; then dAkk =
//      -tril(A^T dA A^T); a second pass per key slab recomputes dQg, dKd, dW
//      and d(gl) from the value slices and runs the score backward per
//      32-channel block (as k_bwd_intra does); the pre-norm dq, dk go to an
//      fp32 section of the workspace and a last pass applies the l2norm
//      backward along each whole row.
// VN and dVN are kept row-major ([64][V]) between these kernels.
#include "chunk_args.cuh"
#include "inverse.cuh"

namespace gdn2 {

namespace {

constexpr int kSlab = 64;            // key / value channels per slab
constexpr int kMaxHead = 256;        // largest K and V served
constexpr int LDW = kSlab + 4;       // row stride of 64 x 64 fp32 slabs
constexpr int LDCW = kChunk + 4;     // row stride of 64 x 64 chunk matrices
constexpr int LDBW = kBV + 4;        // row stride of 32-column tiles

__device__ __forceinline__ float exp2c(float x) { return exp2f(fminf(x, 120.f)); }

// ---------------------------------------------------------------------------
// forward intra
// ---------------------------------------------------------------------------
struct WideIntraSmem {
  static constexpr int oAqk = 0;
  static constexpr int oAkk = oAqk + kChunk * LDCW;
  static constexpr int oG = oAkk + kChunk * LDCW;
  static constexpr int oQ = oG + kChunk * LDW;
  static constexpr int oK = oQ + kChunk * LDW;
  static constexpr int oKB = oK + kChunk * LDW;
  static constexpr int oX = oKB + kChunk * LDW;
  static constexpr int oL = oX + kChunk * LDW;   // [32][LDW]
  static constexpr int oRq = oL + 32 * LDW;
  static constexpr int oRk = oRq + kChunk;
  static constexpr int oTmp = oRk + kChunk;       // 768 floats
  static constexpr int floats = oTmp + 3 * 256;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_fwd_intra_wide(FwdIntraArgs a) {
  using S = WideIntraSmem;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sAqk = sm + S::oAqk;
  float* sAkk = sm + S::oAkk;
  float* sG = sm + S::oG;
  float* sQ = sm + S::oQ;
  float* sK = sm + S::oK;
  float* sKB = sm + S::oKB;
  float* sX = sm + S::oX;
  float* sL = sm + S::oL;
  float* rq = sm + S::oRq;
  float* rk = sm + S::oRk;
  float* tmp = sm + S::oTmp;

  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, K = a.K, V = a.V;
  const ChunkPos cp = chunk_pos(a.seqs, c);
  const int len = cp.len;
  const int64_t ldk = (int64_t)H * K, ldv = (int64_t)H * V;
  const int64_t offk = cp.row0 * ldk + (int64_t)h * K;
  const int64_t offv = cp.row0 * ldv + (int64_t)h * V;
  const T* gq = reinterpret_cast<const T*>(a.q) + offk;
  const T* gk = reinterpret_cast<const T*>(a.k) + offk;
  const T* gb = reinterpret_cast<const T*>(a.b) + offk;
  const float* gg = a.g + offk;
  const T* gv = reinterpret_cast<const T*>(a.v) + offv;
  const T* gw = reinterpret_cast<const T*>(a.w) + offv;
  const size_t ch = (size_t)c * H + h;
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  T* gQg = reinterpret_cast<T*>(a.saved + a.L.qg) + ch * tileK;
  T* gKd = reinterpret_cast<T*>(a.saved + a.L.kd) + ch * tileK;
  T* gW = reinterpret_cast<T*>(a.saved + a.L.w) + ch * tileK;
  T* gU = reinterpret_cast<T*>(a.saved + a.L.u) + ch * tileV;
  T* gAqk = reinterpret_cast<T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk;
  T* gA = reinterpret_cast<T*>(a.saved + a.L.a) + ch * kChunk * kChunk;
  float* gGl = reinterpret_cast<float*>(a.saved + a.L.gl) + ch * K;

  // row norms of q and k over every key channel
  for (int r = warp; r < kChunk; r += kThreads / 32) {
    float sq = 0.f, sk = 0.f;
    if (r < len) {
      for (int cc = lane; cc < K; cc += 32) {
        const float x = to_f<T>(gq[(int64_t)r * ldk + cc]);
        const float y = to_f<T>(gk[(int64_t)r * ldk + cc]);
        sq += x * x;
        sk += y * y;
      }
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      rq[r] = a.l2norm ? rsqrtf(sq + kNormEps) : 1.f;
      rk[r] = a.l2norm ? rsqrtf(sk + kNormEps) : 1.f;
    }
  }
  for (int i = tid; i < kChunk * LDCW; i += kThreads) {
    sAqk[i] = 0.f;
    sAkk[i] = 0.f;
  }
  __syncthreads();

  // G (log2 chunk cumsum), normalised k (and q), b*k_n for key slab c0
  auto load_key_slab = [&](int c0, int nk, bool need_q) {
    load_tile<float, kChunk, kSlab>(sG, LDW, gg + c0, ldk, len, nk);
    if (need_q) load_tile<T, kChunk, kSlab>(sQ, LDW, gq + c0, ldk, len, nk);
    load_tile<T, kChunk, kSlab>(sK, LDW, gk + c0, ldk, len, nk);
    load_tile<T, kChunk, kSlab>(sKB, LDW, gb + c0, ldk, len, nk);
    __syncthreads();
    col_cumsum64<kSlab>(sG, LDW, kLog2e, tmp);
    for (int i = tid; i < kChunk * kSlab; i += kThreads) {
      const int r = i >> 6, cc = i & 63;
      const float kn = sK[r * LDW + cc] * rk[r];
      sK[r * LDW + cc] = kn;
      sKB[r * LDW + cc] *= kn;
      if (need_q) sQ[r * LDW + cc] *= rq[r];
    }
    __syncthreads();
  };

  // ---- scores, Qg, Kd, gl: one key slab at a time --------------------------
  for (int c0 = 0; c0 < K; c0 += kSlab) {
    const int nk = min(kSlab, K - c0);
    load_key_slab(c0, nk, true);
    // off-diagonal blocks: rows of block-row I against keys i < 16 I
    for (int bI = 1; bI < 4; ++bI) {
      const int r0 = 16 * bI;
      for (int i = tid; i < 16 * kSlab; i += kThreads) {
        const int rr = i >> 6, cc = i & 63;
        const float f = exp2c(sG[(r0 + rr) * LDW + cc] - sG[r0 * LDW + cc]);
        sL[rr * LDW + cc] = sQ[(r0 + rr) * LDW + cc] * f;
        sL[(16 + rr) * LDW + cc] = sKB[(r0 + rr) * LDW + cc] * f;
      }
      for (int i = tid; i < r0 * kSlab; i += kThreads) {
        const int ii = i >> 6, cc = i & 63;
        sX[ii * LDW + cc] = sK[ii * LDW + cc] * exp2c(sG[r0 * LDW + cc] - sG[ii * LDW + cc]);
      }
      __syncthreads();
      const int nitems = 2 * bI;  // 2 row tiles (q side, k side) x bI column tiles
      for (int it = warp; it < nitems; it += kThreads / 32) {
        const int mt = it & 1, nt = it >> 1;
        float acc[1][2][4];
        acc_zero(acc);
        warp_mma<1, 2, P>(acc, sL + mt * 16 * LDW, LDW, 1, sX + nt * 16 * LDW, 1, LDW, kSlab);
        acc_foreach(acc, [&](int rr, int cc, float val) {
          const int row = r0 + rr, col = nt * 16 + cc;
          if (mt == 0)
            sAqk[row * LDCW + col] += a.scale * val;
          else
            sAkk[row * LDCW + col] += val;
        });
      }
      __syncthreads();
    }
    // diagonal blocks, exact: 2^(G_r - G_i) per element
    for (int idx = tid; idx < 4 * 256; idx += kThreads) {
      const int bI = idx >> 8, e = idx & 255, rr = e >> 4, ii = e & 15;
      if (ii > rr) continue;
      const int r = 16 * bI + rr, i = 16 * bI + ii;
      float sq = 0.f, skk = 0.f;
      for (int cc = 0; cc < kSlab; ++cc) {
        const float f = exp2c(sG[r * LDW + cc] - sG[i * LDW + cc]) * sK[i * LDW + cc];
        sq += sQ[r * LDW + cc] * f;
        skk += sKB[r * LDW + cc] * f;
      }
      sAqk[r * LDCW + i] += a.scale * sq;
      if (ii < rr) sAkk[r * LDCW + i] += skk;
    }
    for (int i = tid; i < kChunk * kSlab; i += kThreads) {
      const int r = i >> 6, cc = i & 63;
      if (cc < nk) {
        const float G = sG[r * LDW + cc], GL = sG[(kChunk - 1) * LDW + cc];
        gQg[(size_t)r * K + c0 + cc] = from_f<T>(a.scale * sQ[r * LDW + cc] * exp2c(G));
        gKd[(size_t)r * K + c0 + cc] = from_f<T>(sK[r * LDW + cc] * exp2c(GL - G));
      }
    }
    for (int i = tid; i < nk; i += kThreads) gGl[c0 + i] = exp2c(sG[(kChunk - 1) * LDW + i]);
    __syncthreads();
  }
  for (int i = tid; i < kChunk * kChunk; i += kThreads)
    gAqk[i] = from_f<T>(sAqk[(i >> 6) * LDCW + (i & 63)]);
  __syncthreads();

  // ---- A = (I + Akk)^-1 (into sAqk's buffer) ------------------------------
  float* sA = sAqk;
  unit_lower_inverse<LDCW>(sAkk, sA, tmp);
  for (int i = tid; i < kChunk * kChunk; i += kThreads)
    gA[i] = from_f<T>(sA[(i >> 6) * LDCW + (i & 63)]);

  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 32;
  // ---- W = A E, E = b k_n 2^G, per key slab ---------------------------------
  for (int c0 = 0; c0 < K; c0 += kSlab) {
    const int nk = min(kSlab, K - c0);
    load_key_slab(c0, nk, false);
    for (int i = tid; i < kChunk * kSlab; i += kThreads) {
      const int r = i >> 6, cc = i & 63;
      sKB[r * LDW + cc] *= exp2c(sG[r * LDW + cc]);
    }
    __syncthreads();
    float acc[1][4][4];
    acc_zero(acc);
    warp_mma<1, 4, P>(acc, sA + m0 * LDCW, LDCW, 1, sKB + n0, LDW, 1, kChunk);
    acc_foreach(acc, [&](int rr, int cc, float val) {
      const int r = m0 + rr, col = n0 + cc;
      if (col < nk) gW[(size_t)r * K + c0 + col] = from_f<T>(val);
    });
    __syncthreads();
  }
  // ---- U = A Z, Z = w v, per value slab ------------------------------------
  for (int v0 = 0; v0 < V; v0 += kSlab) {
    const int nv = min(kSlab, V - v0);
    load_tile<T, kChunk, kSlab>(sQ, LDW, gv + v0, ldv, len, nv);
    load_tile<T, kChunk, kSlab>(sK, LDW, gw + v0, ldv, len, nv);
    __syncthreads();
    for (int i = tid; i < kChunk * kSlab; i += kThreads) {
      const int r = i >> 6, cc = i & 63;
      sQ[r * LDW + cc] *= sK[r * LDW + cc];
    }
    __syncthreads();
    float acc[1][4][4];
    acc_zero(acc);
    warp_mma<1, 4, P>(acc, sA + m0 * LDCW, LDCW, 1, sQ + n0, LDW, 1, kChunk);
    acc_foreach(acc, [&](int rr, int cc, float val) {
      const int r = m0 + rr, col = n0 + cc;
      if (col < nv) gU[(size_t)r * V + v0 + col] = from_f<T>(val);
    });
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// state passes
// ---------------------------------------------------------------------------
struct WideStateSmem {
  static constexpr int oH = 0;                          // [256][LDBW] state tile
  static constexpr int oA = oH + kMaxHead * LDBW;       // [64][LDW] Qg slab
  static constexpr int oB = oA + kChunk * LDW;          // [64][LDW] W / Kd slab
  static constexpr int oAqk = oB + kChunk * LDW;        // [64][LDCW]
  static constexpr int oU = oAqk + kChunk * LDCW;       // [64][LDBW] U / dO
  static constexpr int oVN = oU + kChunk * LDBW;        // [64][LDBW] VN / dVN
  static constexpr int oGl = oVN + kChunk * LDBW;       // [256]
  static constexpr int floats = oGl + kMaxHead;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_fwd_state_wide(FwdStateArgs a) {
  using S = WideStateSmem;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sH = sm + S::oH;
  float* sQg = sm + S::oA;
  float* sB = sm + S::oB;
  float* sAqk = sm + S::oAqk;
  float* sU = sm + S::oU;
  float* sVN = sm + S::oVN;
  float* sGl = sm + S::oGl;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int H = a.H, K = a.K, V = a.V;
  const int nh = blockIdx.y, n = nh / H, h = nh - n * H;
  const int v0 = blockIdx.x * kBV;
  const int Vx = a.prescan ? V + K : V;  // carried columns
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];

  for (int idx = tid; idx < kMaxHead * kBV; idx += kThreads) {
    const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
    float x = 0.f;
    if (r < K && col < Vx) {
      if (a.prescan)
        x = (col >= V && col - V == r) ? 1.f : 0.f;
      else if (a.h0)
        x = a.h0[(((int64_t)n * H + h) * K + r) * V + col];
    }
    sH[r * LDBW + cc] = x;
  }

  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const int64_t ldo = (int64_t)H * V;
  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 16;
  for (int c = c_begin; c < c_end; ++c) {
    const size_t ch = (size_t)c * H + h;
    const T* gQg = reinterpret_cast<const T*>(a.saved + a.L.qg) + ch * tileK;
    const T* gKd = reinterpret_cast<const T*>(a.saved + a.L.kd) + ch * tileK;
    const T* gW = reinterpret_cast<const T*>(a.saved + a.L.w) + ch * tileK;
    const T* gU = reinterpret_cast<const T*>(a.saved + a.L.u) + ch * tileV;
    const T* gAqk = reinterpret_cast<const T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk;
    const float* gGl = reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K;
    __syncthreads();  // the previous chunk's readers of sU, sAqk, sGl are done
    if (!a.prescan) {
      // checkpoint of the state entering this chunk (for the backward)
      T* gh = reinterpret_cast<T*>(a.saved + a.L.h) + ch * (size_t)K * V;
      for (int idx = tid; idx < K * kBV; idx += kThreads) {
        const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gh[(size_t)r * V + col] = from_f<T>(sH[r * LDBW + cc]);
      }
      load_tile<T, kChunk, kChunk>(sAqk, LDCW, gAqk, kChunk, kChunk, kChunk);
    }
    // U tile (columns beyond V are the M part of the pre-scan: zero)
    load_tile<T, kChunk, kBV>(sU, LDBW, gU + v0, V, kChunk, max(0, min(kBV, V - v0)));
    for (int idx = tid; idx < kMaxHead; idx += kThreads) sGl[idx] = idx < K ? gGl[idx] : 0.f;

    // VN = U - W h,  o = Qg h (+ Aqk VN below): sums over key slabs
    float accV[1][2][4], accO[1][2][4];
    acc_zero(accV);
    acc_zero(accO);
    for (int c0 = 0; c0 < K; c0 += kSlab) {
      const int nk = min(kSlab, K - c0);
      __syncthreads();
      load_tile<T, kChunk, kSlab>(sB, LDW, gW + c0, K, kChunk, nk);
      if (!a.prescan) load_tile<T, kChunk, kSlab>(sQg, LDW, gQg + c0, K, kChunk, nk);
      __syncthreads();
      warp_mma<1, 2, P>(accV, sB + m0 * LDW, LDW, 1, sH + c0 * LDBW + n0, LDBW, 1, kSlab);
      if (!a.prescan)
        warp_mma<1, 2, P>(accO, sQg + m0 * LDW, LDW, 1, sH + c0 * LDBW + n0, LDBW, 1, kSlab);
    }
    acc_foreach(accV, [&](int rr, int cc, float val) {
      const int r = m0 + rr, col = n0 + cc;
      sVN[r * LDBW + col] = sU[r * LDBW + col] - val;
    });
    __syncthreads();
    if (!a.prescan) {
      T* gVN = reinterpret_cast<T*>(a.saved + a.L.vn) + ch * tileV;
      for (int idx = tid; idx < kChunk * kBV; idx += kThreads) {
        const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gVN[(size_t)r * V + col] = from_f<T>(sVN[r * LDBW + cc]);
      }
      const ChunkPos cp = chunk_pos(a.seqs, c);
      warp_mma<1, 2, P>(accO, sAqk + m0 * LDCW, LDCW, 1, sVN + n0, LDBW, 1, kChunk);
      T* go = reinterpret_cast<T*>(a.o) + cp.row0 * ldo + (int64_t)h * V;
      acc_foreach(accO, [&](int rr, int cc, float val) {
        const int r = m0 + rr, col = v0 + n0 + cc;
        if (r < cp.len && col < V) go[r * ldo + col] = from_f<T>(val);
      });
    }
    // h <- gl h + Kd^T VN, one key slab at a time (each warp updates only the
    // state elements of its own tile)
    for (int c0 = 0; c0 < K; c0 += kSlab) {
      const int nk = min(kSlab, K - c0);
      __syncthreads();
      load_tile<T, kChunk, kSlab>(sB, LDW, gKd + c0, K, kChunk, nk);
      __syncthreads();
      float acc[1][2][4];
      acc_zero(acc);
      warp_mma<1, 2, P>(acc, sB + m0, 1, LDW, sVN + n0, LDBW, 1, kChunk);
      acc_foreach(acc, [&](int rr, int cc, float val) {
        const int r = c0 + m0 + rr;
        sH[r * LDBW + n0 + cc] = sGl[r] * sH[r * LDBW + n0 + cc] + val;
      });
    }
  }
  __syncthreads();
  if (a.prescan) {
    for (int idx = tid; idx < K * kBV; idx += kThreads) {
      const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
      if (col < Vx) a.hm[(((int64_t)n * H + h) * K + r) * Vx + col] = sH[r * LDBW + cc];
    }
  } else if (a.ht) {
    for (int idx = tid; idx < K * kBV; idx += kThreads) {
      const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
      if (col < V) a.ht[(((int64_t)n * H + h) * K + r) * V + col] = sH[r * LDBW + cc];
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_bwd_state_wide(BwdStateArgs a) {
  using S = WideStateSmem;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sDH = sm + S::oH;
  float* sA = sm + S::oA;   // Qg slab
  float* sB = sm + S::oB;   // Kd / W slab
  float* sAqk = sm + S::oAqk;
  float* sDO = sm + S::oU;
  float* sDVN = sm + S::oVN;
  float* sGl = sm + S::oGl;

  const int tid = threadIdx.x, warp = tid >> 5;
  const int H = a.H, K = a.K, V = a.V;
  const int nh = blockIdx.y, n = nh / H, h = nh - n * H;
  const int v0 = blockIdx.x * kBV;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];

  for (int idx = tid; idx < kMaxHead * kBV; idx += kThreads) {
    const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
    float x = 0.f;
    if (a.dht && r < K && col < V) x = a.dht[(((int64_t)n * H + h) * K + r) * V + col];
    sDH[r * LDBW + cc] = x;
  }
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const int64_t ldo = (int64_t)H * V;
  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 16;

  for (int c = c_end - 1; c >= c_begin; --c) {
    const size_t ch = (size_t)c * H + h;
    const ChunkPos cp = chunk_pos(a.seqs, c);
    const T* gQg = reinterpret_cast<const T*>(a.saved + a.L.qg) + ch * tileK;
    const T* gKd = reinterpret_cast<const T*>(a.saved + a.L.kd) + ch * tileK;
    const T* gW = reinterpret_cast<const T*>(a.saved + a.L.w) + ch * tileK;
    const float* gGl = reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K;
    __syncthreads();  // the previous chunk's readers of sDO, sAqk, sGl are done
    if (!a.prescan) {
      T* gdh = reinterpret_cast<T*>(a.ws + a.BL.dh) + ch * (size_t)K * V;
      for (int idx = tid; idx < K * kBV; idx += kThreads) {
        const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gdh[(size_t)r * V + col] = from_f<T>(sDH[r * LDBW + cc]);
      }
    }
    load_tile<T, kChunk, kChunk>(sAqk, LDCW,
                                 reinterpret_cast<const T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk,
                                 kChunk, kChunk, kChunk);
    const T* gdo = reinterpret_cast<const T*>(a.dout) + cp.row0 * ldo + (int64_t)h * V + v0;
    load_tile<T, kChunk, kBV>(sDO, LDBW, gdo, ldo, cp.len, min(kBV, V - v0));
    for (int idx = tid; idx < kMaxHead; idx += kThreads) sGl[idx] = idx < K ? gGl[idx] : 0.f;
    __syncthreads();
    // dVN = Aqk^T dO + Kd dh (key slabs)
    float accD[1][2][4];
    acc_zero(accD);
    warp_mma<1, 2, P>(accD, sAqk + m0, 1, LDCW, sDO + n0, LDBW, 1, kChunk);
    for (int c0 = 0; c0 < K; c0 += kSlab) {
      const int nk = min(kSlab, K - c0);
      __syncthreads();
      load_tile<T, kChunk, kSlab>(sB, LDW, gKd + c0, K, kChunk, nk);
      __syncthreads();
      warp_mma<1, 2, P>(accD, sB + m0 * LDW, LDW, 1, sDH + c0 * LDBW + n0, LDBW, 1, kSlab);
    }
    acc_foreach(accD, [&](int rr, int cc, float val) { sDVN[(m0 + rr) * LDBW + n0 + cc] = val; });
    __syncthreads();
    if (!a.prescan) {
      T* gdvn = reinterpret_cast<T*>(a.ws + a.BL.dvn) + ch * tileV;
      for (int idx = tid; idx < kChunk * kBV; idx += kThreads) {
        const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
        if (col < V) gdvn[(size_t)r * V + col] = from_f<T>(sDVN[r * LDBW + cc]);
      }
    }
    // dh <- gl dh + Qg^T dO - W^T dVN, one key slab at a time
    for (int c0 = 0; c0 < K; c0 += kSlab) {
      const int nk = min(kSlab, K - c0);
      __syncthreads();
      load_tile<T, kChunk, kSlab>(sA, LDW, gQg + c0, K, kChunk, nk);
      load_tile<T, kChunk, kSlab>(sB, LDW, gW + c0, K, kChunk, nk);
      __syncthreads();
      float p1[1][2][4], p2[1][2][4];
      acc_zero(p1);
      acc_zero(p2);
      warp_mma<1, 2, P>(p1, sA + m0, 1, LDW, sDO + n0, LDBW, 1, kChunk);
      warp_mma<1, 2, P>(p2, sB + m0, 1, LDW, sDVN + n0, LDBW, 1, kChunk);
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) p1[0][j][e] -= p2[0][j][e];
      acc_foreach(p1, [&](int rr, int cc, float val) {
        const int r = c0 + m0 + rr;
        sDH[r * LDBW + n0 + cc] = sGl[r] * sDH[r * LDBW + n0 + cc] + val;
      });
    }
  }
  __syncthreads();
  if (a.dh0) {
    for (int idx = tid; idx < K * kBV; idx += kThreads) {
      const int r = idx / kBV, cc = idx - r * kBV, col = v0 + cc;
      if (col < V) a.dh0[(((int64_t)n * H + h) * K + r) * V + col] = sDH[r * LDBW + cc];
    }
  }
}

// ---------------------------------------------------------------------------
// backward intra
// ---------------------------------------------------------------------------
struct WideBIntraSmem {
  // persistent
  static constexpr int oA = 0;                        // [64][LDCW] A
  static constexpr int oDAqk = oA + kChunk * LDCW;    // [64][LDCW]
  static constexpr int oDAkk = oDAqk + kChunk * LDCW; // [64][LDCW]
  static constexpr int oT = oDAkk + kChunk * LDCW;    // [64][LDCW] temp
  static constexpr int oDQ = oT + kChunk * LDCW;      // [64][LDW] dQg -> dq (pre-norm), slab
  static constexpr int oDKn = oDQ + kChunk * LDW;     // [64][LDW] dKd -> dk (pre-norm), slab
  static constexpr int oDKB = oDKn + kChunk * LDW;    // [64][LDW] dW -> d(b k), slab
  static constexpr int oRq = oDKB + kChunk * LDW;     // [64]
  static constexpr int oRk = oRq + kChunk;            // [64]
  static constexpr int oDiag = oRk + kChunk;          // [64]
  static constexpr int oPq = oDiag + kChunk;          // [64] q_n . dq partial sums
  static constexpr int oPk = oPq + kChunk;            // [64]
  static constexpr int oDGL = oPk + kChunk;           // [64] d(gl) of the slab
  static constexpr int oGLc = oDGL + kChunk;          // [32]
  static constexpr int oFlag = oGLc + 32;             // [4]
  static constexpr int oR = oFlag + 4;                // work region
  // work region, value slices
  static constexpr int vH = 0, vDH = vH + kChunk * LDBW, vDO = vDH + kChunk * LDBW,
                       vVN = vDO + kChunk * LDBW, vDVN = vVN + kChunk * LDBW,
                       vV = vDVN + kChunk * LDBW, vW = vV + kChunk * LDBW,
                       vZ = vW + kChunk * LDBW, vEnd = vZ + kChunk * LDBW;
  // work region, E of a key slab (G, k, b slabs)
  static constexpr int eG = 0, eK = eG + kChunk * LDW, eB = eK + kChunk * LDW,
                       eEnd = eB + kChunk * LDW;  // + 256 floats of scan scratch
  static_assert(eEnd + 256 <= vEnd, "scan scratch of the E pass fits the work region");
  // work region, 32-channel key blocks
  static constexpr int kq = 0, kk = kq + kChunk * LDBW, kb = kk + kChunk * LDBW,
                       kg = kb + kChunk * LDBW, kx = kg + kChunk * LDBW, ky = kx + kChunk * LDBW,
                       kd = ky + kChunk * LDBW, kl = kd + kChunk * LDBW,
                       kEnd = kl + 32 * LDBW + 256;  // + scan scratch
  static constexpr int region = vEnd > eEnd ? (vEnd > kEnd ? vEnd : kEnd) : (eEnd > kEnd ? eEnd : kEnd);
  static constexpr int floats = oR + region;
  static constexpr size_t bytes = (size_t)floats * sizeof(float);
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) k_bwd_intra_wide(BwdIntraArgs a) {
  using S = WideBIntraSmem;
  constexpr int P = Passes<T>::value;
  extern __shared__ __align__(16) float sm[];
  float* sA = sm + S::oA;
  float* sDAqk = sm + S::oDAqk;
  float* sDAkk = sm + S::oDAkk;
  float* sT = sm + S::oT;
  float* sDQ = sm + S::oDQ;
  float* sDKn = sm + S::oDKn;
  float* sDKB = sm + S::oDKB;
  float* sRq = sm + S::oRq;
  float* sRk = sm + S::oRk;
  float* sDiag = sm + S::oDiag;
  float* sPq = sm + S::oPq;
  float* sPk = sm + S::oPk;
  float* sDGL = sm + S::oDGL;
  float* sGLc = sm + S::oGLc;
  int* sFlag = reinterpret_cast<int*>(sm + S::oFlag);
  float* R = sm + S::oR;
  float* sHs = R + S::vH;
  float* sDHs = R + S::vDH;
  float* sDOs = R + S::vDO;
  float* sVNs = R + S::vVN;
  float* sDVNs = R + S::vDVN;
  float* sVs = R + S::vV;
  float* sWs = R + S::vW;
  float* sZs = R + S::vZ;
  float* sEG = R + S::eG;
  float* sEK = R + S::eK;
  float* sEB = R + S::eB;
  float* sEScan = R + S::eEnd;  // 256 floats past the G, k, b slabs
  float* sCq = R + S::kq;
  float* sCk = R + S::kk;
  float* sCb = R + S::kb;
  float* sCg = R + S::kg;
  float* sCx = R + S::kx;
  float* sCy = R + S::ky;
  float* sCd = R + S::kd;
  float* sCl = R + S::kl;
  float* sScan = sCl + 32 * LDBW;

  const int c = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wr = warp & 3, wc = warp >> 2, m0 = wr * 16;
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
  const T* gh = reinterpret_cast<const T*>(a.saved + a.L.h) + ch * (size_t)K * V;
  const T* gdh = reinterpret_cast<const T*>(a.ws + a.BL.dh) + ch * (size_t)K * V;
  const T* gvn = reinterpret_cast<const T*>(a.saved + a.L.vn) + ch * (size_t)kChunk * V;
  const T* gdvn = reinterpret_cast<const T*>(a.ws + a.BL.dvn) + ch * (size_t)kChunk * V;
  const T* gdo = reinterpret_cast<const T*>(a.dout) + offv;
  const T* gv = reinterpret_cast<const T*>(a.v) + offv;
  const T* gw = reinterpret_cast<const T*>(a.w) + offv;
  const float* gGl = reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K;
  float* wq = reinterpret_cast<float*>(a.ws + a.BL.qk) + ch * 2 * (size_t)kChunk * K;
  float* wk = wq + (size_t)kChunk * K;
  T* gdq = reinterpret_cast<T*>(a.dq) + offk;
  T* gdk = reinterpret_cast<T*>(a.dk) + offk;
  T* gdb = reinterpret_cast<T*>(a.db) + offk;
  float* gdg = a.dg + offk;
  T* gdv = reinterpret_cast<T*>(a.dv) + offv;
  T* gdw = reinterpret_cast<T*>(a.dw) + offv;
  const float scale = a.scale;

  // ---- row norms, A ----------------------------------------------------------
  for (int r = warp; r < kChunk; r += kThreads / 32) {
    float sq = 0.f, sk = 0.f;
    if (r < len) {
      for (int cc = lane; cc < K; cc += 32) {
        const float x = to_f<T>(gq[(int64_t)r * ldk + cc]);
        const float y = to_f<T>(gk[(int64_t)r * ldk + cc]);
        sq += x * x;
        sk += y * y;
      }
    }
    sq = warp_sum(sq);
    sk = warp_sum(sk);
    if (lane == 0) {
      sRq[r] = a.l2norm ? rsqrtf(sq + kNormEps) : 1.f;
      sRk[r] = a.l2norm ? rsqrtf(sk + kNormEps) : 1.f;
      sPq[r] = 0.f;
      sPk[r] = 0.f;
    }
  }
  load_tile<T, kChunk, kChunk>(sA, LDCW,
                               reinterpret_cast<const T*>(a.saved + a.L.a) + ch * kChunk * kChunk,
                               kChunk, kChunk, kChunk);
  __syncthreads();

  // One value slice (32 columns at v0) of the key slab at c0: h and dh rows of
  // the slab, dO, VN, dVN, v, w rows of the chunk.
  auto load_slice = [&](int c0, int nk, int v0, int nv, bool value_rows) {
    load_tile<T, kChunk, kBV>(sHs, LDBW, gh + (size_t)c0 * V + v0, V, nk, nv);
    if (value_rows) {
      load_tile<T, kChunk, kBV>(sDOs, LDBW, gdo + v0, ldv, len, nv);
      load_tile<T, kChunk, kBV>(sDVNs, LDBW, gdvn + v0, V, kChunk, nv);
    }
  };

  // ---- pass 1: dA = dVN Z^T + sum over key slabs of dW E^T; dAqk; dv, dw ----
  float accDA[1][4][4], accAqk[1][4][4];
  acc_zero(accDA);
  acc_zero(accAqk);
  for (int c0 = 0; c0 < K; c0 += kSlab) {
    const int nk = min(kSlab, K - c0);
    const bool first = c0 == 0;
    float accW[1][4][4];
    acc_zero(accW);
    for (int v0 = 0; v0 < V; v0 += kBV) {
      const int nv = min(kBV, V - v0);
      __syncthreads();
      load_slice(c0, nk, v0, nv, true);
      if (first) {
        load_tile<T, kChunk, kBV>(sVNs, LDBW, gvn + v0, V, kChunk, nv);
        load_tile<T, kChunk, kBV>(sVs, LDBW, gv + v0, ldv, len, nv);
        load_tile<T, kChunk, kBV>(sWs, LDBW, gw + v0, ldv, len, nv);
      }
      __syncthreads();
      warp_mma<1, 4, P>(accW, sDVNs + m0 * LDBW, LDBW, 1, sHs + (32 * wc) * LDBW, 1, LDBW, kBV);
      if (first) {
        for (int idx = tid; idx < kChunk * kBV; idx += kThreads) {
          const int r = idx / kBV, cc = idx - r * kBV;
          sZs[r * LDBW + cc] = sVs[r * LDBW + cc] * sWs[r * LDBW + cc];
        }
        __syncthreads();
        warp_mma<1, 4, P>(accAqk, sDOs + m0 * LDBW, LDBW, 1, sVNs + (32 * wc) * LDBW, 1, LDBW,
                          kBV);
        warp_mma<1, 4, P>(accDA, sDVNs + m0 * LDBW, LDBW, 1, sZs + (32 * wc) * LDBW, 1, LDBW,
                          kBV);
        // dZ = A^T dVN -> dv = dZ w, dw = dZ v
        float accZ[1][2][4];
        acc_zero(accZ);
        warp_mma<1, 2, P>(accZ, sA + m0, 1, LDCW, sDVNs + 16 * wc, LDBW, 1, kChunk);
        acc_foreach(accZ, [&](int rr, int cc, float val) {
          const int r = m0 + rr, col = 16 * wc + cc;
          if (r < len && col < nv) {
            gdv[r * ldv + v0 + col] = from_f<T>(val * sWs[r * LDBW + col]);
            gdw[r * ldv + v0 + col] = from_f<T>(val * sVs[r * LDBW + col]);
          }
        });
      }
    }
    __syncthreads();
    // dW of the slab (-dVN h^T) -> sDKB; E = b k_n 2^G of the slab
    acc_foreach(accW, [&](int rr, int cc, float val) { sDKB[(m0 + rr) * LDW + 32 * wc + cc] = -val; });
    load_tile<float, kChunk, kSlab>(sEG, LDW, gg + c0, ldk, len, nk);
    load_tile<T, kChunk, kSlab>(sEK, LDW, gk + c0, ldk, len, nk);
    load_tile<T, kChunk, kSlab>(sEB, LDW, gb + c0, ldk, len, nk);
    __syncthreads();
    col_cumsum64<kSlab>(sEG, LDW, kLog2e, sEScan);
    for (int idx = tid; idx < kChunk * kSlab; idx += kThreads) {
      const int r = idx >> 6, cc = idx & 63;
      sEB[r * LDW + cc] *= sEK[r * LDW + cc] * sRk[r] * exp2c(sEG[r * LDW + cc]);
    }
    __syncthreads();
    warp_mma<1, 4, P>(accDA, sDKB + m0 * LDW, LDW, 1, sEB + (32 * wc) * LDW, 1, LDW, kSlab);
  }
  // dump dAqk (strictly lower; its diagonal kept apart) and dA
  acc_foreach(accAqk, [&](int rr, int cc, float val) {
    const int r = m0 + rr, i = 32 * wc + cc;
    sDAqk[r * LDCW + i] = (i < r) ? val : 0.f;
    if (i == r) sDiag[r] = val;
  });
  acc_foreach(accDA, [&](int rr, int cc, float val) { sT[(m0 + rr) * LDCW + 32 * wc + cc] = val; });
  __syncthreads();
  // dAkk = -tril_strict(A^T dA A^T)
  {
    float t1[1][4][4];
    acc_zero(t1);
    warp_mma<1, 4, P>(t1, sA + m0, 1, LDCW, sT + 32 * wc, LDCW, 1, kChunk);
    __syncthreads();
    acc_foreach(t1, [&](int rr, int cc, float val) { sT[(m0 + rr) * LDCW + 32 * wc + cc] = val; });
    __syncthreads();
    acc_zero(t1);
    warp_mma<1, 4, P>(t1, sT + m0 * LDCW, LDCW, 1, sA + (32 * wc) * LDCW, 1, LDCW, kChunk);
    acc_foreach(t1, [&](int rr, int cc, float val) {
      const int r = m0 + rr, i = 32 * wc + cc;
      sDAkk[r * LDCW + i] = (i < r) ? -val : 0.f;
    });
    __syncthreads();
  }

  // ---- pass 2, per key slab ---------------------------------------------------
  for (int c0s = 0; c0s < K; c0s += kSlab) {
    const int nks = min(kSlab, K - c0s);
    // dQg = dO h^T, dKd = VN dh^T, dW = -dVN h^T over the value slices;
    // d(gl) = rowsum(h * dh)
    float accQ[1][4][4], accKd[1][4][4], accW[1][4][4];
    acc_zero(accQ);
    acc_zero(accKd);
    acc_zero(accW);
    if (tid < kChunk) sDGL[tid] = 0.f;
    for (int v0 = 0; v0 < V; v0 += kBV) {
      const int nv = min(kBV, V - v0);
      __syncthreads();
      load_slice(c0s, nks, v0, nv, true);
      load_tile<T, kChunk, kBV>(sDHs, LDBW, gdh + (size_t)c0s * V + v0, V, nks, nv);
      load_tile<T, kChunk, kBV>(sVNs, LDBW, gvn + v0, V, kChunk, nv);
      __syncthreads();
      if (tid < kChunk) {
        float s = 0.f;
        for (int cc = 0; cc < kBV; ++cc) s += sHs[tid * LDBW + cc] * sDHs[tid * LDBW + cc];
        sDGL[tid] += s;
      }
      warp_mma<1, 4, P>(accQ, sDOs + m0 * LDBW, LDBW, 1, sHs + (32 * wc) * LDBW, 1, LDBW, kBV);
      warp_mma<1, 4, P>(accKd, sVNs + m0 * LDBW, LDBW, 1, sDHs + (32 * wc) * LDBW, 1, LDBW, kBV);
      warp_mma<1, 4, P>(accW, sDVNs + m0 * LDBW, LDBW, 1, sHs + (32 * wc) * LDBW, 1, LDBW, kBV);
    }
    __syncthreads();
    acc_foreach(accQ, [&](int rr, int cc, float val) { sDQ[(m0 + rr) * LDW + 32 * wc + cc] = val; });
    acc_foreach(accKd, [&](int rr, int cc, float val) { sDKn[(m0 + rr) * LDW + 32 * wc + cc] = val; });
    acc_foreach(accW, [&](int rr, int cc, float val) { sDKB[(m0 + rr) * LDW + 32 * wc + cc] = -val; });
    __syncthreads();

    // 32-channel key blocks of the slab (k_bwd_intra's key-block pass)
    for (int cb = 0; cb < nks; cb += 32) {
      const int c0 = c0s + cb;           // first channel of the block
      const int nk = min(32, K - c0);
      load_tile<T, kChunk, 32>(sCq, LDBW, gq + c0, ldk, len, nk);
      load_tile<T, kChunk, 32>(sCk, LDBW, gk + c0, ldk, len, nk);
      load_tile<T, kChunk, 32>(sCb, LDBW, gb + c0, ldk, len, nk);
      load_tile<float, kChunk, 32>(sCg, LDBW, gg + c0, ldk, len, nk);
      __syncthreads();
      for (int idx = tid; idx < kChunk * 32; idx += kThreads) {
        const int r = idx >> 5, cc = idx & 31;
        sCk[r * LDBW + cc] *= sRk[r];
        sCq[r * LDBW + cc] *= sRq[r];
      }
      col_cumsum64<32>(sCg, LDBW, kLog2e, sScan);
      if (tid == 0) sFlag[0] = 1;
      __syncthreads();
      for (int idx = tid; idx < 4 * 32; idx += kThreads) {
        const int bI = idx >> 5, cc = idx & 31;
        const float rng = sCg[(16 * bI) * LDBW + cc] - sCg[(16 * bI + 15) * LDBW + cc];
        if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
      }
      // dE = A^T dW for this block (64 x 32): warp tile 16 x 16
      float accE[1][2][4];
      acc_zero(accE);
      warp_mma<1, 2, P>(accE, sA + m0, 1, LDCW, sDKB + cb + 16 * wc, LDW, 1, kChunk);
      __syncthreads();
      const bool safe = sFlag[0] != 0;
      acc_foreach(accE, [&](int rr, int cc, float val) {
        const int r = m0 + rr, col = 16 * wc + cc;
        sDKB[r * LDW + cb + col] = val * exp2c(sCg[r * LDBW + col]);
      });
      // dq <- scale 2^G dQg;  Kd part of dk <- dKd 2^(G_L - G);  its dG share
      // X_r = k_r (Kd part)_r, shifted one row down for the prefix scan
      for (int idx = tid; idx < kChunk * 32; idx += kThreads) {
        const int r = idx >> 5, cc = idx & 31;
        const float G = sCg[r * LDBW + cc], GL = sCg[(kChunk - 1) * LDBW + cc];
        sDQ[r * LDW + cb + cc] *= scale * exp2c(G);
        const float kdv = sDKn[r * LDW + cb + cc] * exp2c(GL - G);
        sDKn[r * LDW + cb + cc] = kdv;
        if (r + 1 < kChunk) sCy[(r + 1) * LDBW + cc] = sCk[r * LDBW + cc] * kdv;
        if (r == 0) sCy[cc] = 0.f;
        sCd[r * LDBW + cc] = 0.f;
      }
      if (tid < 32) {
        const float gl = (tid < nk) ? gGl[c0 + tid] : 0.f;
        sGLc[tid] = sDGL[cb + tid] * gl;
      }
      // score blocks
      for (int bI = 0; bI < 4; ++bI) {
        const int r0 = 16 * bI, ni = 16 * (bI + 1);
        const int jmax = safe ? ni : 16 * bI;
        __syncthreads();
        for (int idx = tid; idx < 16 * 32; idx += kThreads) {
          const int rr = idx >> 5, cc = idx & 31, r = r0 + rr;
          const float f = exp2c(sCg[r * LDBW + cc] - sCg[r0 * LDBW + cc]);
          sCl[rr * LDBW + cc] = scale * sCq[r * LDBW + cc] * f;
          sCl[(16 + rr) * LDBW + cc] = sCb[r * LDBW + cc] * sCk[r * LDBW + cc] * f;
        }
        for (int idx = tid; idx < ni * 32; idx += kThreads) {
          const int i = idx >> 5, cc = idx & 31;
          sCx[i * LDBW + cc] = sCk[i * LDBW + cc] * exp2c(sCg[r0 * LDBW + cc] - sCg[i * LDBW + cc]);
        }
        __syncthreads();
        if (jmax > 0) {
          {
            const int which = warp >> 2, nt = warp & 3;
            float acc[1][1][4];
            acc_zero(acc);
            warp_mma<1, 1, P>(acc, (which ? sDAkk : sDAqk) + r0 * LDCW, LDCW, 1, sCx + 8 * nt,
                              LDBW, 1, jmax);
            acc_foreach(acc, [&](int rr, int cc, float val) {
              const int r = r0 + rr, col = 8 * nt + cc;
              const float f = exp2c(sCg[r * LDBW + col] - sCg[r0 * LDBW + col]);
              if (which == 0)
                sDQ[r * LDW + cb + col] += scale * val * f;
              else
                sDKB[r * LDW + cb + col] += val * f;
            });
          }
          const int nitems = (jmax / 16) * 4;
          for (int it = warp; it < nitems; it += kThreads / 32) {
            const int mt = it >> 2, nt = it & 3;
            float acc[1][1][4];
            acc_zero(acc);
            warp_mma<1, 1, P>(acc, sDAqk + r0 * LDCW + 16 * mt, 1, LDCW, sCl + 8 * nt, LDBW, 1, 16);
            warp_mma<1, 1, P>(acc, sDAkk + r0 * LDCW + 16 * mt, 1, LDCW, sCl + 16 * LDBW + 8 * nt,
                              LDBW, 1, 16);
            acc_foreach(acc, [&](int rr, int cc, float val) {
              const int i = 16 * mt + rr, col = 8 * nt + cc;
              sCd[i * LDBW + col] += val * exp2c(sCg[r0 * LDBW + col] - sCg[i * LDBW + col]);
            });
          }
        }
        if (!safe) {
          __syncthreads();
          for (int idx = tid; idx < 16 * 32; idx += kThreads) {
            const int rr = idx >> 5, cc = idx & 31, r = r0 + rr;
            float sq = 0.f, sk = 0.f, sy = 0.f;
            for (int ii = 0; ii < rr; ++ii) {
              const int i = r0 + ii;
              const float e = exp2c(sCg[r * LDBW + cc] - sCg[i * LDBW + cc]) * sCk[i * LDBW + cc];
              sq += sDAqk[r * LDCW + i] * e;
              sk += sDAkk[r * LDCW + i] * e;
            }
            for (int r2 = rr + 1; r2 < 16; ++r2) {
              const int rb = r0 + r2;
              const float e = exp2c(sCg[rb * LDBW + cc] - sCg[r * LDBW + cc]);
              const float t = scale * sDAqk[rb * LDCW + r] * sCq[rb * LDBW + cc] +
                              sDAkk[rb * LDCW + r] * sCb[rb * LDBW + cc] * sCk[rb * LDBW + cc];
              sy += t * e;
            }
            sDQ[r * LDW + cb + cc] += scale * sq;
            sDKB[r * LDW + cb + cc] += sk;
            sCd[r * LDBW + cc] += sy;
          }
        }
      }
      __syncthreads();
      // per-element chain: dG (without the Kd part and the diagonal), db, dk
      for (int idx = tid; idx < kChunk * 32; idx += kThreads) {
        const int r = idx >> 5, cc = idx & 31;
        const float qn = sCq[r * LDBW + cc], kn = sCk[r * LDBW + cc], bb = sCb[r * LDBW + cc];
        const float dqn = sDQ[r * LDW + cb + cc], dkb = sDKB[r * LDW + cb + cc];
        const float dy = sCd[r * LDBW + cc];
        float dG = qn * dqn + bb * kn * dkb - kn * dy;
        if (r == len - 1) dG += sGLc[cc];
        sCx[r * LDBW + cc] = dG;
        const float dgn = scale * sDiag[r];
        const float dqf = dqn + dgn * kn;
        const float dkf = sDKn[r * LDW + cb + cc] + dy + dkb * bb + dgn * qn;
        sDQ[r * LDW + cb + cc] = dqf;
        sDKn[r * LDW + cb + cc] = dkf;
        if (r < len && cc < nk) {
          gdb[(int64_t)r * ldk + c0 + cc] = from_f<T>(dkb * kn);
          wq[(size_t)r * K + c0 + cc] = dqf;
          wk[(size_t)r * K + c0 + cc] = dkf;
        }
      }
      __syncthreads();
      // q_n . dq and k_n . dk over this block's channels, for the l2norm backward
      for (int r = warp; r < kChunk; r += kThreads / 32) {
        const float x = sCq[r * LDBW + lane] * sDQ[r * LDW + cb + lane];
        const float y = sCk[r * LDBW + lane] * sDKn[r * LDW + cb + lane];
        const float sx = warp_sum(x), sy = warp_sum(y);
        if (lane == 0) {
          sPq[r] += sx;
          sPk[r] += sy;
        }
      }
      // dg_t = sum_{r>=t} dG_r + sum_{r<t} X_r
      col_scan64<32, true>(sCx, LDBW, sScan);
      col_scan64<32, false>(sCy, LDBW, sScan);
      for (int idx = tid; idx < kChunk * 32; idx += kThreads) {
        const int r = idx >> 5, cc = idx & 31;
        if (r < len && cc < nk)
          gdg[(int64_t)r * ldk + c0 + cc] = sCx[r * LDBW + cc] + sCy[r * LDBW + cc];
      }
      __syncthreads();
    }
  }
  __syncthreads();  // every row's partial sums and pre-norm values are written

  // ---- l2norm backward over whole rows: dx = (dx_n - x_n (x_n . dx_n)) r ----
  for (int r = warp; r < len; r += kThreads / 32) {
    const float rqr = sRq[r], rkr = sRk[r], pq = sPq[r], pk = sPk[r];
    for (int cc = lane; cc < K; cc += 32) {
      float dqv = wq[(size_t)r * K + cc], dkv = wk[(size_t)r * K + cc];
      if (a.l2norm) {
        dqv = (dqv - to_f<T>(gq[(int64_t)r * ldk + cc]) * rqr * pq) * rqr;
        dkv = (dkv - to_f<T>(gk[(int64_t)r * ldk + cc]) * rkr * pk) * rkr;
      }
      gdq[(int64_t)r * ldk + cc] = from_f<T>(dqv);
      gdk[(int64_t)r * ldk + cc] = from_f<T>(dkv);
    }
  }
}

template <typename K_, typename Args>
cudaError_t launch_smem(K_ kern, dim3 grid, size_t bytes, const Args& a, cudaStream_t st) {
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess) return e;
  if (grid.x == 0 || grid.y == 0) return cudaSuccess;
  kern<<<grid, kThreads, bytes, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t launch_fwd_intra_wide(const FwdIntraArgs& a, cudaStream_t st) {
  return launch_smem(k_fwd_intra_wide<T>, dim3(a.seqs.n_chunks, a.H), WideIntraSmem::bytes, a, st);
}
template <typename T>
cudaError_t launch_fwd_state_wide(const FwdStateArgs& a, cudaStream_t st) {
  const int cols = a.prescan ? a.V + a.K : a.V;
  return launch_smem(k_fwd_state_wide<T>, dim3((cols + kBV - 1) / kBV, a.seqs.n_seqs * a.H),
                     WideStateSmem::bytes, a, st);
}
template <typename T>
cudaError_t launch_bwd_state_wide(const BwdStateArgs& a, cudaStream_t st) {
  return launch_smem(k_bwd_state_wide<T>, dim3((a.V + kBV - 1) / kBV, a.seqs.n_seqs * a.H),
                     WideStateSmem::bytes, a, st);
}
template <typename T>
cudaError_t launch_bwd_intra_wide(const BwdIntraArgs& a, cudaStream_t st) {
  return launch_smem(k_bwd_intra_wide<T>, dim3(a.seqs.n_chunks, a.H), WideBIntraSmem::bytes, a,
                     st);
}

#define GDN2_INST_WIDE(T)                                                                  \
  template cudaError_t launch_fwd_intra_wide<T>(const FwdIntraArgs&, cudaStream_t);       \
  template cudaError_t launch_fwd_state_wide<T>(const FwdStateArgs&, cudaStream_t);       \
  template cudaError_t launch_bwd_state_wide<T>(const BwdStateArgs&, cudaStream_t);       \
  template cudaError_t launch_bwd_intra_wide<T>(const BwdIntraArgs&, cudaStream_t);
GDN2_INST_WIDE(float)
GDN2_INST_WIDE(__nv_bfloat16)
GDN2_INST_WIDE(__half)

}  // namespace gdn2
