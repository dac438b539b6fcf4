// state16.cu -- inter-chunk state passes for bf16 inputs.
//
// One CTA of 16 warps per (sequence, head, BV-column value tile) walks the
// sequence's chunks in order (forward) or in reverse (backward).  The fp32
// state tile (D x BV) stays in registers for the whole walk, distributed as
// the accumulator of the state-update product; a 16-bit copy in shared
// memory feeds the products that read it.  The next chunk's per-chunk tiles
// (W, Kd, Qg, Aqk, U or dO, gl) stream in with cp.async into the other half
// of a double buffer while the current chunk computes.  All products are
// mma.sync m16n8k16 with fp32 accumulation from ldmatrix fragments.
//
// forward, per chunk:   VN = U - W h;  o = Qg h + Aqk VN;  h <- gl*h + Kd^T VN
// backward, per chunk:  dVN = Aqk^T dO + Kd dh;  dh <- gl*dh + Qg^T dO - W^T dVN
// (pre-scan modes: the forward carries [h | M] from [0 | I] with no output;
//  the backward keeps only the span-start gradient.)
#include "chunk_args.cuh"
#include "mma16.cuh"

namespace gdn2 {

constexpr int kThreads16 = 512;  // 16 warps

template <int D, int BV>
struct State16Smem {
  static constexpr int LDK = D + 8;       // 64 x D tiles (16-bit)
  static constexpr int LDV = BV + 8;      // 64 x BV and D x BV tiles
  static constexpr int LDC = kChunk + 8;  // 64 x 64 tiles
  static constexpr int buf = 3 * kChunk * LDK + kChunk * LDC + kChunk * LDV;  // elements
  static constexpr size_t bytes16 = (size_t)(2 * buf + D * LDV + kChunk * LDV) * 2;
  static constexpr size_t bytes = bytes16 + 2 * D * sizeof(float);
};

// ---------------------------------------------------------------------------
template <typename T, int D, int BV>
__global__ void __launch_bounds__(kThreads16, 1) k_fwd_state16(FwdStateArgs a) {
  using S = State16Smem<D, BV>;
  constexpr int LDK = S::LDK, LDV = S::LDV, LDC = S::LDC;
  constexpr int MT2 = D / 64, NT2 = BV / 32;  // state tile per warp: (16*MT2) x (8*NT2)
  constexpr int NT1 = BV / 32;                // 64 x BV products: 16 x (8*NT1) per warp
  extern __shared__ __align__(16) unsigned char smraw[];
  T* base = reinterpret_cast<T*>(smraw);
  T* sH = base + 2 * S::buf;            // [D][LDV]
  T* sVN = sH + D * LDV;                // [64][LDV]
  float* sGl = reinterpret_cast<float*>(smraw + S::bytes16);  // [2][D]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int H = a.H, K = a.K, V = a.V;
  const int nh = blockIdx.y, n = nh / H, h = nh - n * H;
  const int v0 = blockIdx.x * BV;
  const int Vx = a.prescan ? V + K : V;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];
  const int64_t bos = a.seqs.cu[n], eos = a.seqs.cu[n + 1];
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const int64_t ldo = (int64_t)H * V;
  const int nU = max(0, min(BV, V - v0));  // U columns present in this tile

  // warp tiles
  const int wm1 = (warp & 3) * 16, wn1 = (warp >> 2) * (BV / 4);            // 64 x BV
  const int wm2 = (warp & 3) * (D / 4), wn2 = (warp >> 2) * (BV / 4);       // D x BV

  auto tiles = [&](int slot) {
    T* p = base + slot * S::buf;
    return p;
  };
  auto issue = [&](int c, int slot) {
    const size_t ch = (size_t)c * H + h;
    T* p = tiles(slot);
    T* sW = p;
    T* sKd = sW + kChunk * LDK;
    T* sQg = sKd + kChunk * LDK;
    T* sAqk = sQg + kChunk * LDK;
    T* sU = sAqk + kChunk * LDC;
    cp_tile16<T, kChunk, D, kThreads16>(sW, LDK, reinterpret_cast<const T*>(a.saved + a.L.w) +
                                                      ch * tileK, K, kChunk, K);
    cp_tile16<T, kChunk, D, kThreads16>(sKd, LDK, reinterpret_cast<const T*>(a.saved + a.L.kd) +
                                                       ch * tileK, K, kChunk, K);
    if (!a.prescan) {
      cp_tile16<T, kChunk, D, kThreads16>(
          sQg, LDK, reinterpret_cast<const T*>(a.saved + a.L.qg) + ch * tileK, K, kChunk, K);
      cp_tile16<T, kChunk, kChunk, kThreads16>(
          sAqk, LDC, reinterpret_cast<const T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk, kChunk,
          kChunk, kChunk);
    }
    cp_tile16<T, kChunk, BV, kThreads16>(
        sU, LDV, reinterpret_cast<const T*>(a.saved + a.L.u) + ch * tileV + (nU > 0 ? v0 : 0), V,
        kChunk, nU);
    cp_vec32<D, kThreads16>(sGl + slot * D,
                            reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K, K);
    cp_async_commit();
  };

  // ---- initial state (registers + 16-bit copy) ----------------------------
  float hreg[MT2][NT2][4];
#pragma unroll
  for (int i = 0; i < MT2; ++i)
#pragma unroll
    for (int j = 0; j < NT2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = wm2 + 16 * i + gid + ((e >> 1) << 3);
        const int col = v0 + wn2 + 8 * j + 2 * tig + (e & 1);
        float x = 0.f;
        if (r < K && col < Vx) {
          if (a.prescan)
            x = (col >= V && col - V == r) ? 1.f : 0.f;
          else if (a.h0)
            x = a.h0[(((int64_t)n * H + h) * K + r) * V + col];
        }
        hreg[i][j][e] = x;
      }
  auto store_state16 = [&]() {
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = wm2 + 16 * i + gid + 8 * hf;
          const int cl = wn2 + 8 * j + 2 * tig;
          *reinterpret_cast<uint32_t*>(sH + r * LDV + cl) =
              pack2<T>(hreg[i][j][2 * hf], hreg[i][j][2 * hf + 1]);
        }
  };
  auto store_ckpt = [&](int c) {
    T* gh = reinterpret_cast<T*>(a.saved + a.L.h) + ((size_t)c * H + h) * (size_t)K * V;
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = wm2 + 16 * i + gid + 8 * hf;
          const int col = v0 + wn2 + 8 * j + 2 * tig;
          if (r < K && col < V)
            *reinterpret_cast<uint32_t*>(gh + (size_t)r * V + col) =
                pack2<T>(hreg[i][j][2 * hf], hreg[i][j][2 * hf + 1]);
        }
  };
  store_state16();
  if (c_begin < c_end) issue(c_begin, 0);

  for (int c = c_begin; c < c_end; ++c) {
    const int slot = (c - c_begin) & 1;
    if (c + 1 < c_end) {
      issue(c + 1, slot ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    if (!a.prescan) store_ckpt(c);
    __syncthreads();  // tiles of chunk c and sH visible
    T* sW = tiles(slot);
    T* sKd = sW + kChunk * LDK;
    T* sQg = sKd + kChunk * LDK;
    T* sAqk = sQg + kChunk * LDK;
    T* sU = sAqk + kChunk * LDC;
    const float* gl = sGl + slot * D;
    const size_t ch = (size_t)c * H + h;

    // VN = U - W h
    {
      float acc[1][NT1][4];
      acc_zero(acc);
      warp_mma16<1, NT1, true, false>(acc, sW, LDK, wm1, sH, LDV, wn1, D);
      T* gVN = reinterpret_cast<T*>(a.saved + a.L.vn) + ch * tileV;
#pragma unroll
      for (int j = 0; j < NT1; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = wm1 + gid + 8 * hf;
          const int cl = wn1 + 8 * j + 2 * tig;
          const float u0 = to_f<T>(sU[r * LDV + cl]), u1 = to_f<T>(sU[r * LDV + cl + 1]);
          const float x0 = u0 - acc[0][j][2 * hf], x1 = u1 - acc[0][j][2 * hf + 1];
          const uint32_t pk = pack2<T>(x0, x1);
          *reinterpret_cast<uint32_t*>(sVN + r * LDV + cl) = pk;
          if (!a.prescan && v0 + cl < V) {  // saved VN^T: [V][64]
            gVN[(size_t)(v0 + cl) * kChunk + r] = from_f<T>(x0);
            if (v0 + cl + 1 < V) gVN[(size_t)(v0 + cl + 1) * kChunk + r] = from_f<T>(x1);
          }
        }
    }
    __syncthreads();  // sVN visible
    // o = Qg h + Aqk VN
    if (!a.prescan) {
      const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);
      float acc[1][NT1][4];
      acc_zero(acc);
      warp_mma16<1, NT1, true, false>(acc, sQg, LDK, wm1, sH, LDV, wn1, D);
      warp_mma16<1, NT1, true, false>(acc, sAqk, LDC, wm1, sVN, LDV, wn1, kChunk);
      T* go = reinterpret_cast<T*>(a.o) + cp.row0 * ldo + (int64_t)h * V;
#pragma unroll
      for (int j = 0; j < NT1; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = wm1 + gid + 8 * hf;
          const int col = v0 + wn1 + 8 * j + 2 * tig;
          if (r < cp.len && col < V)
            *reinterpret_cast<uint32_t*>(go + r * ldo + col) =
                pack2<T>(acc[0][j][2 * hf], acc[0][j][2 * hf + 1]);
        }
    }
    // h <- gl*h + Kd^T VN  (accumulated into the register state)
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) hreg[i][j][e] *= gl[wm2 + 16 * i + gid + ((e >> 1) << 3)];
    warp_mma16<MT2, NT2, false, false>(hreg, sKd, LDK, wm2, sVN, LDV, wn2, kChunk);
    __syncthreads();  // all reads of sH / sVN / this slot are done
    store_state16();
  }

  // final state
  float* out = a.prescan ? a.hm : a.ht;
  const int ld_out = a.prescan ? Vx : V;
  if (out) {
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = wm2 + 16 * i + gid + ((e >> 1) << 3);
          const int col = v0 + wn2 + 8 * j + 2 * tig + (e & 1);
          if (r < K && col < Vx) out[(((int64_t)n * H + h) * K + r) * ld_out + col] = hreg[i][j][e];
        }
  }
}

// ---------------------------------------------------------------------------
template <typename T, int D, int BV>
__global__ void __launch_bounds__(kThreads16, 1) k_bwd_state16(BwdStateArgs a) {
  using S = State16Smem<D, BV>;
  constexpr int LDK = S::LDK, LDV = S::LDV, LDC = S::LDC;
  constexpr int MT2 = D / 64, NT2 = BV / 32;
  constexpr int NT1 = BV / 32;
  extern __shared__ __align__(16) unsigned char smraw[];
  T* base = reinterpret_cast<T*>(smraw);
  T* sDH = base + 2 * S::buf;           // [D][LDV]
  T* sNDVN = sDH + D * LDV;             // [64][LDV]  -dVN
  float* sGl = reinterpret_cast<float*>(smraw + S::bytes16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int H = a.H, K = a.K, V = a.V;
  const int nh = blockIdx.y, n = nh / H, h = nh - n * H;
  const int v0 = blockIdx.x * BV;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];
  const int64_t bos = a.seqs.cu[n], eos = a.seqs.cu[n + 1];
  const size_t tileK = (size_t)kChunk * K, tileV = (size_t)kChunk * V;
  const int64_t ldo = (int64_t)H * V;
  const int nV = max(0, min(BV, V - v0));
  const int wm1 = (warp & 3) * 16, wn1 = (warp >> 2) * (BV / 4);
  const int wm2 = (warp & 3) * (D / 4), wn2 = (warp >> 2) * (BV / 4);

  auto tiles = [&](int slot) { return base + slot * S::buf; };
  auto issue = [&](int c, int slot) {
    const size_t ch = (size_t)c * H + h;
    const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);
    T* sW = tiles(slot);
    T* sKd = sW + kChunk * LDK;
    T* sQg = sKd + kChunk * LDK;
    T* sAqk = sQg + kChunk * LDK;
    T* sDO = sAqk + kChunk * LDC;
    cp_tile16<T, kChunk, D, kThreads16>(sW, LDK, reinterpret_cast<const T*>(a.saved + a.L.w) +
                                                      ch * tileK, K, kChunk, K);
    cp_tile16<T, kChunk, D, kThreads16>(sKd, LDK, reinterpret_cast<const T*>(a.saved + a.L.kd) +
                                                       ch * tileK, K, kChunk, K);
    cp_tile16<T, kChunk, D, kThreads16>(sQg, LDK, reinterpret_cast<const T*>(a.saved + a.L.qg) +
                                                       ch * tileK, K, kChunk, K);
    cp_tile16<T, kChunk, kChunk, kThreads16>(
        sAqk, LDC, reinterpret_cast<const T*>(a.saved + a.L.aqk) + ch * kChunk * kChunk, kChunk,
        kChunk, kChunk);
    cp_tile16<T, kChunk, BV, kThreads16>(
        sDO, LDV, reinterpret_cast<const T*>(a.dout) + cp.row0 * ldo + (int64_t)h * V + v0, ldo,
        cp.len, nV);
    cp_vec32<D, kThreads16>(sGl + slot * D,
                            reinterpret_cast<const float*>(a.saved + a.L.gl) + ch * K, K);
    cp_async_commit();
  };

  float dh[MT2][NT2][4];
#pragma unroll
  for (int i = 0; i < MT2; ++i)
#pragma unroll
    for (int j = 0; j < NT2; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = wm2 + 16 * i + gid + ((e >> 1) << 3);
        const int col = v0 + wn2 + 8 * j + 2 * tig + (e & 1);
        dh[i][j][e] = (a.dht && r < K && col < V)
                          ? a.dht[(((int64_t)n * H + h) * K + r) * V + col] : 0.f;
      }
  auto store_state16 = [&]() {
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = wm2 + 16 * i + gid + 8 * hf;
          const int cl = wn2 + 8 * j + 2 * tig;
          *reinterpret_cast<uint32_t*>(sDH + r * LDV + cl) =
              pack2<T>(dh[i][j][2 * hf], dh[i][j][2 * hf + 1]);
        }
  };
  store_state16();
  if (c_begin < c_end) issue(c_end - 1, 0);

  for (int c = c_end - 1; c >= c_begin; --c) {
    const int slot = (c_end - 1 - c) & 1;
    if (c - 1 >= c_begin) {
      issue(c - 1, slot ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    const size_t ch = (size_t)c * H + h;
    if (!a.prescan) {
      // gradient w.r.t. the state leaving chunk c
      T* gdh = reinterpret_cast<T*>(a.ws + a.BL.dh) + ch * (size_t)K * V;
#pragma unroll
      for (int i = 0; i < MT2; ++i)
#pragma unroll
        for (int j = 0; j < NT2; ++j)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int r = wm2 + 16 * i + gid + 8 * hf;
            const int col = v0 + wn2 + 8 * j + 2 * tig;
            if (r < K && col < V)
              *reinterpret_cast<uint32_t*>(gdh + (size_t)r * V + col) =
                  pack2<T>(dh[i][j][2 * hf], dh[i][j][2 * hf + 1]);
          }
    }
    __syncthreads();
    T* sW = tiles(slot);
    T* sKd = sW + kChunk * LDK;
    T* sQg = sKd + kChunk * LDK;
    T* sAqk = sQg + kChunk * LDK;
    T* sDO = sAqk + kChunk * LDC;
    const float* gl = sGl + slot * D;

    // dVN = Aqk^T dO + Kd dh
    {
      float acc[1][NT1][4];
      acc_zero(acc);
      warp_mma16<1, NT1, false, false>(acc, sAqk, LDC, wm1, sDO, LDV, wn1, kChunk);
      warp_mma16<1, NT1, true, false>(acc, sKd, LDK, wm1, sDH, LDV, wn1, D);
      T* gdvn = reinterpret_cast<T*>(a.ws + a.BL.dvn) + ch * tileV;
#pragma unroll
      for (int j = 0; j < NT1; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = wm1 + gid + 8 * hf;
          const int cl = wn1 + 8 * j + 2 * tig;
          const float x0 = acc[0][j][2 * hf], x1 = acc[0][j][2 * hf + 1];
          *reinterpret_cast<uint32_t*>(sNDVN + r * LDV + cl) = pack2<T>(-x0, -x1);
          if (!a.prescan && v0 + cl < V) {  // dVN^T: [V][64]
            gdvn[(size_t)(v0 + cl) * kChunk + r] = from_f<T>(x0);
            if (v0 + cl + 1 < V) gdvn[(size_t)(v0 + cl + 1) * kChunk + r] = from_f<T>(x1);
          }
        }
    }
    __syncthreads();
    // dh <- gl*dh + Qg^T dO + W^T (-dVN)
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) dh[i][j][e] *= gl[wm2 + 16 * i + gid + ((e >> 1) << 3)];
    warp_mma16<MT2, NT2, false, false>(dh, sQg, LDK, wm2, sDO, LDV, wn2, kChunk);
    warp_mma16<MT2, NT2, false, false>(dh, sW, LDK, wm2, sNDVN, LDV, wn2, kChunk);
    __syncthreads();
    store_state16();
  }

  if (a.dh0) {
#pragma unroll
    for (int i = 0; i < MT2; ++i)
#pragma unroll
      for (int j = 0; j < NT2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = wm2 + 16 * i + gid + ((e >> 1) << 3);
          const int col = v0 + wn2 + 8 * j + 2 * tig + (e & 1);
          if (r < K && col < V) a.dh0[(((int64_t)n * H + h) * K + r) * V + col] = dh[i][j][e];
        }
  }
}

// ---------------------------------------------------------------------------
template <typename T, int D, int BV>
cudaError_t launch_fwd_state16(const FwdStateArgs& a, cudaStream_t st) {
  auto kern = k_fwd_state16<T, D, BV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)State16Smem<D, BV>::bytes);
  if (e != cudaSuccess) return e;
  const int cols = a.prescan ? a.V + a.K : a.V;
  dim3 grid((cols + BV - 1) / BV, a.seqs.n_seqs * a.H);
  kern<<<grid, kThreads16, State16Smem<D, BV>::bytes, st>>>(a);
  return cudaGetLastError();
}

template <typename T, int D, int BV>
cudaError_t launch_bwd_state16(const BwdStateArgs& a, cudaStream_t st) {
  auto kern = k_bwd_state16<T, D, BV>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)State16Smem<D, BV>::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid((a.V + BV - 1) / BV, a.seqs.n_seqs * a.H);
  kern<<<grid, kThreads16, State16Smem<D, BV>::bytes, st>>>(a);
  return cudaGetLastError();
}

#define GDN2_INST_STATE16(T, D, BV)                                                       \
  template cudaError_t launch_fwd_state16<T, D, BV>(const FwdStateArgs&, cudaStream_t);  \
  template cudaError_t launch_bwd_state16<T, D, BV>(const BwdStateArgs&, cudaStream_t);
GDN2_INST_STATE16(__nv_bfloat16, 64, 64)
GDN2_INST_STATE16(__nv_bfloat16, 128, 64)
GDN2_INST_STATE16(__nv_bfloat16, 128, 128)

}  // namespace gdn2
