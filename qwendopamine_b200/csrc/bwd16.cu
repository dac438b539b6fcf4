// bwd16.cu -- per-chunk GDN-2 gradients for bf16 inputs.
//
// One CTA of 16 warps per (chunk, head).  Same mathematics as k_bwd_intra
// (chunk_bwd.cu), organised so that almost nothing waits on memory:
//   * every tile arrives by TMA, requested by one thread (issuing the copies
//     thread by thread with cp.async kept the CTA waiting on the load queue):
//     q, k, b (16-bit), g (fp32) and A once;
//   * the value side streams 32-column slices of h, dh, dO, VN, dVN, v, w
//     (VN and dVN are stored value-major, [V][64], by the bf16 state passes)
//     through a two-slot buffer while the previous slice computes
//     (dQg = dO h^T, dKd = VN dh^T, dW = -dVN h^T, dAqk = dO VN^T,
//      dA = dVN (w v)^T, dZ = A^T dVN -> dv, dw);
//   * the key side needs no further loads.  Each warp owns a 16-row x D/4
//     column tile and keeps its dq, d(b k), dk, dG and Kd-term accumulators
//     in registers; the score backward products are issued so that their
//     outputs land on the owning warp (block-row I of the X products on the
//     warps of row block I, block-column J of the Y products on those of J).
// All products: ldmatrix fragments, mma.sync m16n8k16, fp32 accumulation.
// As in k_bwd_intra, the dAqk diagonal and the last-row Kd term are kept out
// of dG (they cancel exactly), and dg is a suffix scan of dG plus a prefix
// scan of the Kd terms.
#include "chunk_args.cuh"
#include "mma16.cuh"
#include "tc.cuh"

namespace gdn2 {

constexpr int kThreadsB16 = 512;

template <int D, bool TC = false>
struct Bwd16Layout {
  static constexpr int LDK = D + 8;      // 16-bit 64 x D tiles
  static constexpr int LDG = D + 8;      // fp32 64 x D tiles (8-byte pairs conflict-free)
  static constexpr int LDC = kChunk + 8; // 16-bit 64 x 64 tiles
  static constexpr int LDS = 32 + 8;     // 16-bit value slices
  static constexpr int LDT = kChunk + 8; // 16-bit VN^T / dVN^T slices [32][64]
  // persistent region (bytes)
  static constexpr int oQ = 0;
  static constexpr int oK = oQ + kChunk * LDK * 2;
  static constexpr int oB = oK + kChunk * LDK * 2;
  static constexpr int oG = oB + kChunk * LDK * 2;
  static constexpr int oA = oG + kChunk * LDG * 4;
  static constexpr int oMisc = oA + kChunk * LDC * 2;
  // misc floats: rq[64] rk[64] dgl[D] diag[64] pdq[4][64] pdk[4][64] flag[4] F[10][D]
  //              dApart[16], then 3 mbarriers (as 6 floats, 8-byte aligned)
  static constexpr int nMisc = 64 + 64 + D + 64 + 256 + 256 + 4 + 10 * D + 16;
  // TMA targets: 128-byte aligned; 1024 with the tcgen05 value phase, whose
  // 128-byte-swizzled tiles need it (and 4 mbarriers + the TMEM address)
  static constexpr int oW = TC ? (oMisc + nMisc * 4 + 6 * 8 + 1023) / 1024 * 1024
                               : (oMisc + nMisc * 4 + 3 * 8 + 127) / 128 * 128;
  // phase V (offsets inside W)
  static constexpr int vH = 0;
  static constexpr int vDH = vH + D * LDS * 2;
  static constexpr int vDO = vDH + D * LDS * 2;
  static constexpr int vVN = vDO + kChunk * LDS * 2;
  static constexpr int vDVN = vVN + kChunk * LDS * 2;
  static constexpr int vV = vDVN + kChunk * LDS * 2;
  static constexpr int vWg = vV + kChunk * LDS * 2;
  static constexpr int slot = vWg + kChunk * LDS * 2;
  static constexpr int vZ = 2 * slot;
  static constexpr int phaseV = vZ + kChunk * LDS * 2;
  // phase K
  static constexpr int kDAqk = 0;
  static constexpr int kDAkk = kDAqk + kChunk * LDC * 2;
  static constexpr int kR2 = kDAkk + kChunk * LDC * 2;
  static constexpr int kDW = kR2;
  static constexpr int kE = kDW + kChunk * LDK * 2;
  static constexpr int kT1 = kE + kChunk * LDK * 2;
  static constexpr int kT2 = kT1 + kChunk * LDC * 2;
  static constexpr int kQs = kR2;
  static constexpr int kKBs = kQs + kChunk * LDK * 2;
  static constexpr int kKb = kKBs + kChunk * LDK * 2;
  static constexpr int kEnd = kKb + kChunk * LDK * 2;
  static constexpr int kdG = 0;
  static constexpr int kX = kdG + kChunk * LDG * 4;
  static constexpr int kTmp = kX + kChunk * LDG * 4;
  static constexpr int kScanEnd = kTmp + 4 * kThreadsB16 * 4;
  // tcgen05 value phase (K = V = 128): two 64-column slices of 128-byte-
  // swizzled tiles; h / dh [128][64] single-buffered, dO, VN^T, dVN^T, v, w
  // [64][64] in two slots, Z = v w; after it, a fp32 [64][LDG] transpose
  // buffer at kE and the scan scratch beyond it
  static constexpr int tH = 0, tDH = 16384, tSlot0 = 32768, tSlotBytes = 40960;
  static constexpr int tDO = 0, tVN = 8192, tDVN = 16384, tV = 24576, tWg = 32768;
  static constexpr int tZ = tSlot0 + 2 * tSlotBytes;
  static constexpr int tEnd = tZ + 8192;
  static constexpr int tTr = kE;
  // the Kd terms X (fp32 [64][LDG], shifted down one row) wait here from the
  // owner initialisation until the dg scan, clear of the score operands and
  // of the scan's own tiles
  static constexpr int tXs = (kScanEnd + 1023) / 1024 * 1024;
  static constexpr int tScan = (tTr + kChunk * LDG * 4 + 1023) / 1024 * 1024;
  static constexpr int W0 = phaseV > kEnd ? (phaseV > kScanEnd ? phaseV : kScanEnd)
                                          : (kEnd > kScanEnd ? kEnd : kScanEnd);
  static constexpr int Wtc = tEnd > tScan + 4 * kThreadsB16 ? tEnd : tScan + 4 * kThreadsB16;
  static constexpr int W = TC ? (W0 > Wtc ? W0 : Wtc) : W0;
  static constexpr size_t bytes = (size_t)oW + W + (TC ? 1024 : 128);  // + base alignment slack
  static_assert(kT2 + kChunk * LDC * 2 <= kEnd || kT2 + kChunk * LDC * 2 <= W, "layout");
  static_assert(oW % 128 == 0 && slot % 128 == 0 && oK % 128 == 0 && oB % 128 == 0 &&
                    oG % 128 == 0 && oA % 128 == 0 && vDH % 128 == 0 && vDO % 128 == 0 &&
                    vVN % 128 == 0 && vDVN % 128 == 0 && vV % 128 == 0 && vWg % 128 == 0,
                "TMA destinations are 128-byte aligned");
  static_assert((oMisc + nMisc * 4) % 8 == 0, "mbarrier alignment");
  static_assert(32 * LDT <= kChunk * LDS, "VN^T slice fits its region");
  static_assert(3 * kChunk * LDK * 2 <= W, "gradient staging fits the work region");
  static_assert(!TC || D == 128, "the tcgen05 value phase serves K = V = 128");
  static_assert(!TC || (tTr >= kDW + kChunk * LDK * 2), "transpose buffer clear of dW");
  static_assert(!TC || bytes <= 232448, "shared memory per CTA");
  static_assert(!TC || tXs + kChunk * LDG * 4 <= W, "X tile fits the work region");
  static_assert(!TC || tXs >= kEnd, "X tile clear of the score operands");
};

// TMA views of every tile the kernel reads (built per launch on the host).
struct Bwd16Maps {
  CUtensorMap q, k, b, g;       // [rows][H][K] token rows (g fp32)
  CUtensorMap a, h, dh;         // per (chunk, head): A [64][64], h / dh [K][V]
  CUtensorMap dout, v, w;       // [rows][H][V] token rows
  CUtensorMap vn, dvn;          // per (chunk, head): VN / dVN stored [V][64]
};

template <typename T, int D, bool TC>
__global__ void __launch_bounds__(kThreadsB16, 1)
    k_bwd_intra16(BwdIntraArgs a, const __grid_constant__ Bwd16Maps mp) {
  using L = Bwd16Layout<D, TC>;
  constexpr int LDK = L::LDK, LDG = L::LDG, LDC = L::LDC, LDS = L::LDS, LDT = L::LDT;
  constexpr int NTH = kThreadsB16;
  constexpr int DQ = D / 4;    // owner tile width
  constexpr int NTO = DQ / 8;  // n8 fragments per owner tile
  extern __shared__ unsigned char smraw[];
  constexpr uint32_t kAlign = TC ? 1024u : 128u;
  unsigned char* sm = smraw + ((kAlign - (smem_u32(smraw) & (kAlign - 1))) & (kAlign - 1));
  T* sq = reinterpret_cast<T*>(sm + L::oQ);
  T* sk = reinterpret_cast<T*>(sm + L::oK);
  T* sb = reinterpret_cast<T*>(sm + L::oB);
  float* sG = reinterpret_cast<float*>(sm + L::oG);
  T* sA = reinterpret_cast<T*>(sm + L::oA);
  float* misc = reinterpret_cast<float*>(sm + L::oMisc);
  float* rq = misc;
  float* rk = rq + 64;
  float* dgl = rk + 64;
  float* sDiag = dgl + D;
  float* pdq = sDiag + 64;  // [4][64]
  float* pdk = pdq + 256;   // [4][64]
  int* sFlag = reinterpret_cast<int*>(pdk + 256);
  float* sF = pdk + 256 + 4;  // [10][D] 2^(G_16I - G_(16J+15)), pair I(I+1)/2 + J
  float* sDApart = sF + 10 * D;  // [16] per-warp dL/dA_log partial sums (gate in kernel)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDApart + 16);  // [0], [1] slots, [2] q k b g
  unsigned char* W = sm + L::oW;

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

  // Every tile arrives by TMA (one thread issues, the others keep computing)
  // as a box whose rows are as wide as the padded shared-memory rows, so the
  // pad columns come along (or read as zero past the tensor's edge).  Slices
  // of the value side complete on the mbarrier of their slot, q, k, b, g on
  // a third.  Rows past a partial chunk's end hold the next sequence's
  // tokens and are zeroed after landing.
  const int nslices = (V + 31) / 32;
  const int crow = (int)cp.row0;
  const uint32_t txSlice = (uint32_t)(2 * LDS * 2 * K + 3 * LDS * 2 * kChunk + 2 * LDT * 2 * 32);
  const uint32_t txA = (uint32_t)(LDC * 2 * kChunk);
  const uint32_t txKey = (uint32_t)(3 * LDK * 2 * kChunk + LDG * 4 * kChunk);
  auto slotp = [&](int s, int off) { return reinterpret_cast<T*>(W + s * L::slot + off); };
  auto issue_slice = [&](int v0, int s) {  // thread 0
    tc::tma_load_2d(slotp(s, L::vH), &mp.h, v0, (int)ch * K, &bars[s]);
    tc::tma_load_2d(slotp(s, L::vDH), &mp.dh, v0, (int)ch * K, &bars[s]);
    tc::tma_load_3d(slotp(s, L::vDO), &mp.dout, v0, h, crow, &bars[s]);
    tc::tma_load_2d(slotp(s, L::vVN), &mp.vn, 0, (int)ch * V + v0, &bars[s]);
    tc::tma_load_2d(slotp(s, L::vDVN), &mp.dvn, 0, (int)ch * V + v0, &bars[s]);
    tc::tma_load_3d(slotp(s, L::vV), &mp.v, v0, h, crow, &bars[s]);
    tc::tma_load_3d(slotp(s, L::vWg), &mp.w, v0, h, crow, &bars[s]);
  };
  // The value side needs only A and the value slices; q, k, b, g (key side)
  // are requested after the next-slice copies (q with slice 1, k and b with
  // slice 2, g with slice 3; all remaining ones with the last) so their
  // latency hides behind the value-side products.
  auto issue_key_part = [&](int part) {  // thread 0
    if (part == 0) {
      tc::tma_load_3d(sq, &mp.q, 0, h, crow, &bars[2]);
    } else if (part == 1) {
      tc::tma_load_3d(sk, &mp.k, 0, h, crow, &bars[2]);
      tc::tma_load_3d(sb, &mp.b, 0, h, crow, &bars[2]);
    } else {
      tc::tma_load_3d(sG, &mp.g, 0, h, crow, &bars[2]);
    }
  };
  // rows [r0, r1) of a tile of 16-byte-multiple rows (generic-proxy zeros)
  auto zero_rows = [&](void* t, int row_bytes, int r0, int r1) {
    const int n16 = row_bytes / 16;
    for (int e = tid; e < (r1 - r0) * n16; e += NTH) {
      const int r = r0 + e / n16, c = e - (e / n16) * n16;
      reinterpret_cast<uint4*>(static_cast<unsigned char*>(t) + (size_t)r * row_bytes)[c] =
          make_uint4(0u, 0u, 0u, 0u);
    }
  };
  // A wait that ran out: let the copies still in flight land (bounded),
  // flag the fault and leave.
  // (slices 0 .. last_slice have been requested; slice t fills slot t & 1 in
  // that slot's phase t >> 1)
  auto drain = [&](int last_slice) {
    if (tid == 0) {
      for (int t = last_slice > 1 ? last_slice - 1 : 0; t <= last_slice; ++t)
        tc::mbar_wait(&bars[t & 1], (t >> 1) & 1);
      tc::mbar_wait(&bars[2], 0);
      atomicOr(a.fault, 8u);
    }
  };

  // ---- phase V --------------------------------------------------------------
  float accQ[1][NTO][4], accKd[1][NTO][4], accW[1][NTO][4], accAqk[1][2][4], accDA[1][2][4];
  acc_zero(accQ);
  acc_zero(accKd);
  acc_zero(accW);
  acc_zero(accAqk);
  acc_zero(accDA);
  T* sZ = reinterpret_cast<T*>(W + L::vZ);
  T* gdv = reinterpret_cast<T*>(a.dv) + offv;
  T* gdw = reinterpret_cast<T*>(a.dw) + offv;
  // ---- tcgen05 value phase (K = V = 128) -------------------------------------
  // Two 64-column value slices in 128-byte-swizzled tiles.  One thread issues
  //   dQg^T += h dO^T,  dKd^T += dh VN^T,  dW'^T += h dVN^T   (TMEM cols 0,
  //   64, 128; M = 128 key rows, N = 64 tokens, K = the slice's 64 columns)
  // while the warps form Z = v w and d(gl), the 16 x 16 products dAqk += dO
  // VN^T and dA += dVN Z^T, and dZ = A^T dVN -> dv, dw on mma.sync.  The h /
  // dh tiles of slice 1 replace slice 0's once its products have read them.
  // Afterwards dW goes from TMEM straight to its bf16 tile and dQg, dKd reach
  // the owner-tile registers through one fp32 shared-memory transpose each.
  uint32_t tmem = 0;
  if constexpr (TC) {
    uint64_t* barMma = bars + 3;
    uint32_t* sTmemAddr = reinterpret_cast<uint32_t*>(bars + 4);
    if (tid == 0) {
      for (int i = 0; i < 3; ++i) tc::mbar_init(&bars[i], 1);
      tc::mbar_init(barMma, 3);
      tc::fence_mbar_init();
    }
    if (warp == 0) {
      tc::tmem_alloc(sTmemAddr, 256);
      tc::tmem_relinquish();
    }
    for (int i = tid; i < D; i += NTH) dgl[i] = 0.f;
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    tmem = *sTmemAddr;
    constexpr uint32_t kTxSlice = 2 * 16384 + 5 * 8192;  // h, dh, dO, VN^T, dVN^T, v, w
    auto tp = [&](int off) { return reinterpret_cast<T*>(W + off); };
    auto slot_off = [&](int sl, int off) { return L::tSlot0 + sl * L::tSlotBytes + off; };
    int mma_commits = 0;  // thread 0
    auto drain_tc = [&]() {
      if (tid == 0) {
        for (int i = 0; i < 3; ++i) tc::mbar_wait(&bars[i], 0);
        if (mma_commits > 0) tc::mbar_wait(barMma, (mma_commits - 1) & 1);
        atomicOr(a.fault, 8u);
      }
      tc::tc_fence_before();
      __syncthreads();
      if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 256);
      }
    };
    if (tid == 0) {
      tc::mbar_expect_tx(&bars[0], kTxSlice + txA);
      tc::tma_load_2d(sA, &mp.a, 0, (int)ch * kChunk, &bars[0]);
      tc::tma_load_2d(tp(L::tH), &mp.h, 0, (int)ch * K, &bars[0]);
      tc::tma_load_2d(tp(L::tDH), &mp.dh, 0, (int)ch * K, &bars[0]);
      for (int sl = 0; sl < 2; ++sl) {
        if (sl == 1) tc::mbar_expect_tx(&bars[1], kTxSlice);  // h / dh follow later
        tc::tma_load_3d(tp(slot_off(sl, L::tDO)), &mp.dout, 64 * sl, h, crow, &bars[sl]);
        tc::tma_load_2d(tp(slot_off(sl, L::tVN)), &mp.vn, 0, (int)ch * V + 64 * sl, &bars[sl]);
        tc::tma_load_2d(tp(slot_off(sl, L::tDVN)), &mp.dvn, 0, (int)ch * V + 64 * sl, &bars[sl]);
        tc::tma_load_3d(tp(slot_off(sl, L::tV)), &mp.v, 64 * sl, h, crow, &bars[sl]);
        tc::tma_load_3d(tp(slot_off(sl, L::tWg)), &mp.w, 64 * sl, h, crow, &bars[sl]);
      }
      tc::mbar_expect_tx(&bars[2], txKey);
      for (int part = 0; part < 3; ++part) issue_key_part(part);
    }
    T* th = tp(L::tH);
    T* tdh = tp(L::tDH);
    T* tz = tp(L::tZ);
    // dv / dw of slice sl (staged over its w / v tiles) -> global rows, one
    // 16-byte chunk per thread and tile; callers are past a barrier
    auto copy_dvdw = [&](int sl) {
      const int r = tid >> 3, c = tid & 7;
      if (r < len) {
        const unsigned char* sw_ = reinterpret_cast<const unsigned char*>(tp(slot_off(sl, L::tWg)));
        const unsigned char* sv_ = reinterpret_cast<const unsigned char*>(tp(slot_off(sl, L::tV)));
        const int off = r * 128 + ((c ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(gdv + r * ldv + 64 * sl + 8 * c) =
            *reinterpret_cast<const uint4*>(sw_ + off);
        *reinterpret_cast<uint4*>(gdw + r * ldv + 64 * sl + 8 * c) =
            *reinterpret_cast<const uint4*>(sv_ + off);
      }
    };
    constexpr uint32_t kIdKK = tc::idesc_bf16(128, 64, 0, 0);  // K-major A, K-major B
    constexpr uint32_t kIdKM = tc::idesc_bf16(128, 64, 0, 1);  // K-major A, MN-major B
    for (int sl = 0; sl < 2; ++sl) {
      T* tdo = tp(slot_off(sl, L::tDO));
      T* tvn = tp(slot_off(sl, L::tVN));
      T* tdvn = tp(slot_off(sl, L::tDVN));
      T* tv = tp(slot_off(sl, L::tV));
      T* tw = tp(slot_off(sl, L::tWg));
      if (__syncthreads_or(!tc::mbar_wait(&bars[sl], 0))) {
        drain_tc();
        return;
      }
      if (sl == 1) copy_dvdw(0);
      if (len < kChunk) {  // rows past a partial chunk hold the next sequence's tokens
        zero_rows(tdo, 128, len, kChunk);
        zero_rows(tv, 128, len, kChunk);
        zero_rows(tw, 128, len, kChunk);
        tc::fence_async_smem();
        __syncthreads();
      }
      // lane 0 of warps 0, 1, 2 each issue one product and commit (barMma
      // counts three arrivals), so no warp carries all twelve issues
      if (lane == 0 && warp < 3) {
        tc::tc_fence_after();
        // descriptors: layout constants OR the tile address in 16-byte units
        const uint32_t w16 = smem_u32(W) >> 4, s16 = w16 + (slot_off(sl, 0) >> 4);
        const uint64_t dK = tc::sdesc_layout(16, 1024, tc::kSwizzle128);
        const uint64_t dM = tc::sdesc_layout(8192, 1024, tc::kSwizzle128);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t acc = (sl > 0 || j > 0) ? 1u : 0u;
          if (warp == 0)
            tc::umma_bf16(tmem + 0, dK | (w16 + (L::tH >> 4) + 2 * j),
                          dK | (s16 + (L::tDO >> 4) + 2 * j), kIdKK, acc);
          else if (warp == 1)
            tc::umma_bf16(tmem + 64, dK | (w16 + (L::tDH >> 4) + 2 * j),
                          dM | (s16 + (L::tVN >> 4) + 128 * j), kIdKM, acc);
          else
            tc::umma_bf16(tmem + 128, dK | (w16 + (L::tH >> 4) + 2 * j),
                          dM | (s16 + (L::tDVN >> 4) + 128 * j), kIdKM, acc);
        }
        tc::umma_commit(barMma);
        if (warp == 0) ++mma_commits;
      }
      // Z = v w (same swizzle as v, w): one 16-byte chunk per thread
      {
        const int r = tid >> 3, c = tid & 7;
        const int off = r * 128 + ((c ^ (r & 7)) << 4);
        const uint4 v8 = *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(tv) + off);
        const uint4 w8 = *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(tw) + off);
        uint4 z8;
        float2 p;
        p = mul2(unpack2<T>(v8.x), unpack2<T>(w8.x)); z8.x = pack2<T>(p.x, p.y);
        p = mul2(unpack2<T>(v8.y), unpack2<T>(w8.y)); z8.y = pack2<T>(p.x, p.y);
        p = mul2(unpack2<T>(v8.z), unpack2<T>(w8.z)); z8.z = pack2<T>(p.x, p.y);
        p = mul2(unpack2<T>(v8.w), unpack2<T>(w8.w)); z8.w = pack2<T>(p.x, p.y);
        *reinterpret_cast<uint4*>(reinterpret_cast<unsigned char*>(tz) + off) = z8;
      }
      // dgl[k] += sum over the slice's 64 columns of h * dh: 4 threads per
      // key row, two 16-byte chunks each, combined with two shuffles
      {
        const int row = tid >> 2, part = tid & 3;
        float acc = 0.f;
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int c = 2 * part + q;
          const int off = row * 128 + ((c ^ (row & 7)) << 4);
          const uint4 h8 = *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(th) + off);
          const uint4 d8 = *reinterpret_cast<const uint4*>(reinterpret_cast<const unsigned char*>(tdh) + off);
          float2 acc2 = mul2(unpack2<T>(h8.x), unpack2<T>(d8.x));
          acc2 = fma2(unpack2<T>(h8.y), unpack2<T>(d8.y), acc2);
          acc2 = fma2(unpack2<T>(h8.z), unpack2<T>(d8.z), acc2);
          acc2 = fma2(unpack2<T>(h8.w), unpack2<T>(d8.w), acc2);
          acc += acc2.x + acc2.y;
        }
        acc += __shfl_xor_sync(0xffffffffu, acc, 1);
        acc += __shfl_xor_sync(0xffffffffu, acc, 2);
        if (part == 0) dgl[row] += acc;
      }
      __syncthreads();  // Z is complete; every read of h / dh by the threads is done
      if (sl == 0 && tid == 0) {
        // h / dh of slice 1 once slice 0's products have read them
        if (tc::mbar_wait(barMma, 0)) {
          tc::tma_load_2d(th, &mp.h, 64, (int)ch * K, &bars[1]);
          tc::tma_load_2d(tdh, &mp.dh, 64, (int)ch * K, &bars[1]);
        }
      }
      // dAqk += dO VN^T, dA += dVN Z^T (16 x 16 tiles)
#pragma unroll
      for (int k0 = 0; k0 < 64; k0 += 16) {
        uint32_t aDo[4], aDvn[4], b[4];
        load_a16_sw<true>(aDo, tdo, 16 * wr, k0);
        load_a16_sw<false>(aDvn, tdvn, 16 * wr, k0);
        load_b16x2_sw<false>(b, tvn, k0, 16 * wc);
        Mma16<T>::run(accAqk[0][0], aDo, b[0], b[1]);
        Mma16<T>::run(accAqk[0][1], aDo, b[2], b[3]);
        load_b16x2_sw<true>(b, tz, k0, 16 * wc);
        Mma16<T>::run(accDA[0][0], aDvn, b[0], b[1]);
        Mma16<T>::run(accDA[0][1], aDvn, b[2], b[3]);
      }
      {
        // dZ = A^T dVN (64 tokens x the slice's 64 columns): 16 x 16 per warp
        float accZ[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        const int zm = 16 * (warp & 3), zn = 16 * (warp >> 2);
        const int rr8 = lane & 7, kh = (lane >> 3) & 1;
#pragma unroll
        for (int k0 = 0; k0 < kChunk; k0 += 16) {
          uint32_t af[4];
          load_a16<false>(af, sA, LDC, zm, k0);
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t bf[2];
            ldsm_x2(bf, sw128(tdvn, zn + 8 * h2 + rr8, k0 + 8 * kh));
            Mma16<T>::run(accZ[h2], af, bf[0], bf[1]);
          }
        }
        // dv = dZ w and dw = dZ v replace w and v element by element (each
        // element is read and written by this thread only; nothing else reads
        // v, w after Z); they leave as whole rows after the next barrier
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int r = zm + gid + 8 * hf, cl = zn + 8 * h2 + 2 * tig;
            const float2 z2 = pr(accZ[h2], hf);
            T* pw = const_cast<T*>(sw128_elem(tw, r, cl));
            T* pv = const_cast<T*>(sw128_elem(tv, r, cl));
            const float2 dv2 = mul2(z2, ld2<T>(pw));
            const float2 dw2 = mul2(z2, ld2<T>(pv));
            *reinterpret_cast<uint32_t*>(pw) = pack2<T>(dv2.x, dv2.y);
            *reinterpret_cast<uint32_t*>(pv) = pack2<T>(dw2.x, dw2.y);
          }
      }
    }
    // every product of both slices has landed in TMEM
    if (__syncthreads_or(!tc::warp_wait(barMma, 1))) {
      drain_tc();
      return;
    }
    copy_dvdw(1);  // (slot 1 stays untouched until the owner initialisation)
    tc::tc_fence_after();
    {
      const int q4 = warp & 3, cg = warp >> 2;  // TMEM lanes 32 q4 .., token columns 16 cg ..
      const uint32_t tl = tmem + ((uint32_t)(32 * q4) << 16);
      const int kk = 32 * q4 + lane;            // key channel of this thread's lane
      float* sTr = reinterpret_cast<float*>(W + L::tTr);
      T* sDWt = reinterpret_cast<T*>(W + L::kDW);
      uint32_t x[16];
      tc::tmem_ld16(tl + 128 + 16 * cg, x);
      tc::tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) sDWt[(16 * cg + e) * LDK + kk] = from_f<T>(-__uint_as_float(x[e]));
      tc::tmem_ld16(tl + 0 + 16 * cg, x);
      tc::tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) sTr[(16 * cg + e) * LDG + kk] = __uint_as_float(x[e]);
      __syncthreads();
#pragma unroll
      for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * wr + gid + 8 * hf, c0 = wc * DQ + 8 * j + 2 * tig;
          setpr(accQ[0][j], hf, ld2<float>(sTr + r * LDG + c0));
        }
      __syncthreads();
      tc::tmem_ld16(tl + 64 + 16 * cg, x);
      tc::tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 16; ++e) sTr[(16 * cg + e) * LDG + kk] = __uint_as_float(x[e]);
      __syncthreads();
#pragma unroll
      for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int r = 16 * wr + gid + 8 * hf, c0 = wc * DQ + 8 * j + 2 * tig;
          setpr(accKd[0][j], hf, ld2<float>(sTr + r * LDG + c0));
        }
    }
  } else {
  // ---- phase 0: A and the first slice --------------------------------------
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) tc::mbar_init(&bars[i], 1);
    tc::fence_mbar_init();
  }
  if (K < D) {  // h / dh rows past K are never loaded
    for (int sl = 0; sl < 2; ++sl) {
      zero_rows(slotp(sl, L::vH), LDS * 2, K, D);
      zero_rows(slotp(sl, L::vDH), LDS * 2, K, D);
    }
  }
  for (int i = tid; i < D; i += NTH) dgl[i] = 0.f;
  tc::fence_async_smem();
  __syncthreads();
  if (tid == 0) {
    tc::mbar_expect_tx(&bars[2], txKey);
    tc::mbar_expect_tx(&bars[0], txSlice + txA);
    tc::tma_load_2d(sA, &mp.a, 0, (int)ch * kChunk, &bars[0]);
    issue_slice(0, 0);
    if (nslices == 1)
      for (int part = 0; part < 3; ++part) issue_key_part(part);
  }

  for (int s = 0; s < nslices; ++s) {
    const int cur = s & 1, v0 = 32 * s, nv = min(32, V - v0);
    if (s + 1 < nslices) {
      tc::fence_async_smem();
      __syncthreads();  // the other slot's last readers (and zeroing writers) are done
      if (tid == 0) {
        tc::mbar_expect_tx(&bars[cur ^ 1], txSlice);
        issue_slice(v0 + 32, cur ^ 1);
        if (s + 2 == nslices) {
          for (int part = s; part < 3; ++part) issue_key_part(part);
        } else if (s < 3) {
          issue_key_part(s);
        }
      }
    }
    if (__syncthreads_or(!tc::mbar_wait(&bars[cur], (s >> 1) & 1))) {
      drain(s + 1 < nslices ? s + 1 : s);
      return;
    }
    if (len < kChunk || nv < 32) {
      if (len < kChunk) {
        zero_rows(slotp(cur, L::vDO), LDS * 2, len, kChunk);
        zero_rows(slotp(cur, L::vV), LDS * 2, len, kChunk);
        zero_rows(slotp(cur, L::vWg), LDS * 2, len, kChunk);
      }
      if (nv < 32) {  // VN / dVN rows past the last value column belong to the next head
        zero_rows(slotp(cur, L::vVN), LDT * 2, nv, 32);
        zero_rows(slotp(cur, L::vDVN), LDT * 2, nv, 32);
      }
      __syncthreads();
    }
    T* hs = slotp(cur, L::vH);
    T* dhs = slotp(cur, L::vDH);
    T* dos = slotp(cur, L::vDO);
    T* vns = slotp(cur, L::vVN);
    T* dvns = slotp(cur, L::vDVN);
    T* vs = slotp(cur, L::vV);
    T* ws = slotp(cur, L::vWg);
    // Z = v w: a warp takes rows r and r + 4 (80-byte rows: 32 distinct banks)
    for (int i = tid; i < kChunk * 16; i += NTH) {
      const int b5 = i >> 5, r = (b5 >> 2) * 8 + (b5 & 3) + 4 * ((i >> 4) & 1), cc = (i & 15) * 2;
      const float2 v2 = ld2<T>(vs + r * LDS + cc), w2 = ld2<T>(ws + r * LDS + cc);
      const float2 z2 = mul2(v2, w2);
      *reinterpret_cast<uint32_t*>(sZ + r * LDS + cc) = pack2<T>(z2.x, z2.y);
    }
    // dgl[row] += sum over the slice's 32 columns of h * dh: 4 threads per
    // row, 8 columns each, combined with two shuffles
    for (int i = tid; i < 4 * D; i += NTH) {
      const int row = i >> 2, part = i & 3;
      const uint4 h8 = *reinterpret_cast<const uint4*>(hs + row * LDS + 8 * part);
      const uint4 d8 = *reinterpret_cast<const uint4*>(dhs + row * LDS + 8 * part);
      float2 acc2 = mul2(unpack2<T>(h8.x), unpack2<T>(d8.x));
      acc2 = fma2(unpack2<T>(h8.y), unpack2<T>(d8.y), acc2);
      acc2 = fma2(unpack2<T>(h8.z), unpack2<T>(d8.z), acc2);
      acc2 = fma2(unpack2<T>(h8.w), unpack2<T>(d8.w), acc2);
      float acc = acc2.x + acc2.y;
      acc += __shfl_xor_sync(0xffffffffu, acc, 1);
      acc += __shfl_xor_sync(0xffffffffu, acc, 2);
      if (part == 0) dgl[row] += acc;
    }
    __syncthreads();
    // dQg += dO h^T, dKd += VN dh^T, dW += dVN h^T (owner tiles), dAqk += dO
    // VN^T, dA += dVN Z^T (16 x 16 tiles): each A fragment (dO, dVN, VN) and
    // each B fragment of h loaded once for the products that share it
#pragma unroll
    for (int k0 = 0; k0 < 32; k0 += 16) {
      uint32_t aDo[4], aDvn[4], aVn[4], b[4];
      load_a16<true>(aDo, dos, LDS, 16 * wr, k0);
      load_a16<false>(aDvn, dvns, LDT, 16 * wr, k0);
      load_a16<false>(aVn, vns, LDT, 16 * wr, k0);
#pragma unroll
      for (int j = 0; j < NTO; j += 2) {
        load_b16x2<true>(b, hs, LDS, k0, wc * DQ + 8 * j);
        Mma16<T>::run(accQ[0][j], aDo, b[0], b[1]);
        Mma16<T>::run(accQ[0][j + 1], aDo, b[2], b[3]);
        Mma16<T>::run(accW[0][j], aDvn, b[0], b[1]);
        Mma16<T>::run(accW[0][j + 1], aDvn, b[2], b[3]);
        load_b16x2<true>(b, dhs, LDS, k0, wc * DQ + 8 * j);
        Mma16<T>::run(accKd[0][j], aVn, b[0], b[1]);
        Mma16<T>::run(accKd[0][j + 1], aVn, b[2], b[3]);
      }
      load_b16x2<false>(b, vns, LDT, k0, 16 * wc);
      Mma16<T>::run(accAqk[0][0], aDo, b[0], b[1]);
      Mma16<T>::run(accAqk[0][1], aDo, b[2], b[3]);
      load_b16x2<true>(b, sZ, LDS, k0, 16 * wc);
      Mma16<T>::run(accDA[0][0], aDvn, b[0], b[1]);
      Mma16<T>::run(accDA[0][1], aDvn, b[2], b[3]);
    }
    {
      // Z = A^T dVN (64 tokens x the slice's 32 columns): a 16 x 8 tile per warp
      float accZ[4] = {0.f, 0.f, 0.f, 0.f};
      const int zm = 16 * (warp & 3), zn = 8 * (warp >> 2);
      warp_mma16_n8<false>(accZ, sA, LDC, zm, dvns, LDT, zn, kChunk);
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = zm + gid + 8 * hf, cl = zn + 2 * tig;
        if (r < len && cl < nv) {
          const float2 z2 = pr(accZ, hf);
          const float2 dv2 = mul2(z2, ld2<T>(ws + r * LDS + cl));
          const float2 dw2 = mul2(z2, ld2<T>(vs + r * LDS + cl));
          *reinterpret_cast<uint32_t*>(gdv + r * ldv + v0 + cl) = pack2<T>(dv2.x, dv2.y);
          *reinterpret_cast<uint32_t*>(gdw + r * ldv + v0 + cl) = pack2<T>(dw2.x, dw2.y);
        }
      }
    }
  }
  }
  // phase V buffers are dead from here on; q, k, b, g have landed
  if (__syncthreads_or(!tc::mbar_wait(&bars[2], 0))) {
    if constexpr (TC) {
      if (tid == 0) atomicOr(a.fault, 8u);
      tc::tc_fence_before();
      __syncthreads();
      if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, 256);
      }
    } else {
      drain(nslices - 1);
    }
    return;
  }
  if (len < kChunk) {
    zero_rows(sq, LDK * 2, len, kChunk);
    zero_rows(sk, LDK * 2, len, kChunk);
    zero_rows(sb, LDK * 2, len, kChunk);
    zero_rows(sG, LDG * 4, len, kChunk);
    __syncthreads();
  }
  if (a.gate.mode) {  // gate in kernel: raw input -> log-decay (valid rows / channels)
    for (int i = tid; i < kChunk * D; i += NTH) {
      const int r = i / D, cc = i - r * D;
      if (r < len && cc < K) sG[r * LDG + cc] = gate_apply(a.gate, sG[r * LDG + cc], h, cc, K);
    }
    __syncthreads();
  }
  // chunk-local log2 cumulative decay; row norms
  col_scan64_reg<D, NTH, false>(sG, LDG, reinterpret_cast<float*>(W + (TC ? L::tScan : L::vZ)),
                                kLog2e);
  row_norms16<T, D, NTH>(sq, sk, LDK, rq, rk, a.l2norm);

  // ---- dump dW and dAqk ------------------------------------------------------
  T* sDAqk = reinterpret_cast<T*>(W + L::kDAqk);
  T* sDAkk = reinterpret_cast<T*>(W + L::kDAkk);
  T* sDW = reinterpret_cast<T*>(W + L::kDW);
  T* sE = reinterpret_cast<T*>(W + L::kE);
  T* sT1 = reinterpret_cast<T*>(W + L::kT1);
  T* sT2 = reinterpret_cast<T*>(W + L::kT2);
  if constexpr (!TC) {  // (the tcgen05 value phase wrote sDW from TMEM)
#pragma unroll
    for (int j = 0; j < NTO; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
        *reinterpret_cast<uint32_t*>(sDW + r * LDK + cl) =
            pack2<T>(-accW[0][j][2 * hf], -accW[0][j][2 * hf + 1]);
      }
  }
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf, i0 = 16 * wc + 8 * j + 2 * tig;
      const float x0 = accAqk[0][j][2 * hf], x1 = accAqk[0][j][2 * hf + 1];
      *reinterpret_cast<uint32_t*>(sDAqk + r * LDC + i0) =
          pack2<T>(i0 < r ? x0 : 0.f, i0 + 1 < r ? x1 : 0.f);
      if (i0 == r) sDiag[r] = x0;
      if (i0 + 1 == r) sDiag[r] = x1;
    }
  __syncthreads();  // every warp's row norms are in (the E pass reads all rows)
  // E = b * k_n * 2^G
  for (int i = tid; i < kChunk * (D / 2); i += NTH) {
    const int r = i / (D / 2), cc = (i - r * (D / 2)) * 2;
    const float2 b2 = ld2<T>(sb + r * LDK + cc), k2 = ld2<T>(sk + r * LDK + cc);
    const float2 G2 = ld2<float>(sG + r * LDG + cc);
    const float2 e = mul2(mul2(mul2(b2, k2), f2(rk[r])), exp2_2(G2));
    *reinterpret_cast<uint32_t*>(sE + r * LDK + cc) = pack2<T>(e.x, e.y);
  }
  __syncthreads();
  // dA += dW E^T ; dAkk = -tril_strict(A^T dA A^T)
  warp_mma16<1, 2, true, true>(accDA, sDW, LDK, 16 * wr, sE, LDK, 16 * wc, D);
#pragma unroll
  for (int j = 0; j < 2; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf, cl = 16 * wc + 8 * j + 2 * tig;
      *reinterpret_cast<uint32_t*>(sT1 + r * LDC + cl) =
          pack2<T>(accDA[0][j][2 * hf], accDA[0][j][2 * hf + 1]);
    }
  __syncthreads();
  {
    float t[1][2][4];
    acc_zero(t);
    warp_mma16<1, 2, false, false>(t, sA, LDC, 16 * wr, sT1, LDC, 16 * wc, kChunk);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = 16 * wr + gid + 8 * hf, cl = 16 * wc + 8 * j + 2 * tig;
        *reinterpret_cast<uint32_t*>(sT2 + r * LDC + cl) = pack2<T>(t[0][j][2 * hf], t[0][j][2 * hf + 1]);
      }
    __syncthreads();
    acc_zero(t);
    warp_mma16<1, 2, true, true>(t, sT2, LDC, 16 * wr, sA, LDC, 16 * wc, kChunk);
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int r = 16 * wr + gid + 8 * hf, i0 = 16 * wc + 8 * j + 2 * tig;
        *reinterpret_cast<uint32_t*>(sDAkk + r * LDC + i0) =
            pack2<T>(i0 < r ? -t[0][j][2 * hf] : 0.f, i0 + 1 < r ? -t[0][j][2 * hf + 1] : 0.f);
      }
  }
  // dE = A^T dW (owner tile)
  float accE[1][NTO][4];
  acc_zero(accE);
  warp_mma16<1, NTO, false, false>(accE, sA, LDC, 16 * wr, sDW, LDK, wc * DQ, kChunk);

  // every read of sDW / sE / sT* is done: R2 becomes the score operands
  if (tid == 0) sFlag[0] = 1;
  __syncthreads();

  // ---- owner initialisation and score operands ----------------------------
  // dq <- scale 2^G dQg, dkb <- 2^G dE, dk <- Kd part, X <- k_n * Kd part,
  // dG <- q_n dq + b k_n dkb; in the same pass (same loads) the score
  // backward's operands with per-16-row-block references (every factor <= 1):
  //   Qs[r] = scale q_n[r] 2^(G_r - G_b(r)),  KBs[r] = (b k_n)[r] 2^(G_r - G_b(r)),
  //   Kb[i] = k_n[i] 2^(G_e(i) - G_i);
  // key block J enters block row I scaled by F_IJ = 2^(G_16I - G_(16J+15)).
  float (&dq)[1][NTO][4] = accQ;
  float (&dkb)[1][NTO][4] = accE;
  float (&dkn)[1][NTO][4] = accKd;
  float (&dG)[1][NTO][4] = accW;
  T* sQs = reinterpret_cast<T*>(W + L::kQs);
  T* sKBs = reinterpret_cast<T*>(W + L::kKBs);
  T* sKb = reinterpret_cast<T*>(W + L::kKb);
  block_factors<D, NTH>(sG, LDG, sF);
  // (owner elements come in column pairs: e = 2 hf + t is row 16 wr + gid +
  // 8 hf, column wc DQ + 8 j + 2 tig + t, so each pair is one 32-bit access)
  // The Kd terms X wait for the dg scan in registers, or (tcgen05 layout,
  // fewer live registers through the score backward) in shared memory.
  float X[TC ? 1 : NTO][4];
  float* sXs = reinterpret_cast<float*>(W + (TC ? L::tXs : 0));
#pragma unroll
  for (int j = 0; j < NTO; ++j) {
    const int c0 = wc * DQ + 8 * j + 2 * tig;
    const float2 GL2 = ld2<float>(sG + (kChunk - 1) * LDG + c0);
    const float2 Gb2 = ld2<float>(sG + (16 * wr) * LDG + c0);
    const float2 Ge2 = ld2<float>(sG + (16 * wr + 15) * LDG + c0);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf;
      const float2 G2 = ld2<float>(sG + r * LDG + c0);
      const float2 q2 = ld2<T>(sq + r * LDK + c0), k2 = ld2<T>(sk + r * LDK + c0);
      const float2 b2 = ld2<T>(sb + r * LDK + c0);
      const float2 gam = exp2_2(G2);
      const float2 qn = mul2(q2, f2(rq[r])), kn = mul2(k2, f2(rk[r]));
      const float2 bkn = mul2(b2, kn);
      const float2 dqv = mul2(mul2(f2(scale), gam), pr(dq[0][j], hf));
      const float2 dkbv = mul2(gam, pr(dkb[0][j], hf));
      const float2 kd = mul2(pr(dkn[0][j], hf), exp2_2(make_float2(GL2.x - G2.x, GL2.y - G2.y)));
      setpr(dq[0][j], hf, dqv);
      setpr(dkb[0][j], hf, dkbv);
      setpr(dkn[0][j], hf, kd);
      if constexpr (TC) {
        if (r + 1 < kChunk) *reinterpret_cast<float2*>(sXs + (r + 1) * LDG + c0) = mul2(kn, kd);
      } else {
        setpr(X[j], hf, mul2(kn, kd));
      }
      setpr(dG[0][j], hf, fma2(qn, dqv, mul2(bkn, dkbv)));
      const float2 f = exp2_2(make_float2(G2.x - Gb2.x, G2.y - Gb2.y));
      const float2 fe = exp2_2(make_float2(Ge2.x - G2.x, Ge2.y - G2.y));
      const float2 qs = mul2(mul2(f2(scale), qn), f);
      const float2 kbs = mul2(bkn, f);
      const float2 kb = mul2(kn, fe);
      *reinterpret_cast<uint32_t*>(sQs + r * LDK + c0) = pack2<T>(qs.x, qs.y);
      *reinterpret_cast<uint32_t*>(sKBs + r * LDK + c0) = pack2<T>(kbs.x, kbs.y);
      *reinterpret_cast<uint32_t*>(sKb + r * LDK + c0) = pack2<T>(kb.x, kb.y);
    }
  }
  for (int i = tid; i < 4 * D; i += NTH) {
    const int bI = i / D, cc = i - bI * D;
    const float rng = sG[(16 * bI) * LDG + cc] - sG[(16 * bI + 15) * LDG + cc];
    if (!(rng <= kSafeLog2Range)) sFlag[0] = 0;
  }
  __syncthreads();
  const bool safe = sFlag[0] != 0;
  {
    // X products: rows of block I = wr, one 16-key block J at a time, the
    // owner columns in halves of NXH n8 tiles (fewer live accumulators)
    const int I = wr, nJ = safe ? I + 1 : I;
    if (nJ > 0) {
      constexpr int NXH = NTO >= 4 ? NTO / 2 : NTO;
#pragma unroll
      for (int h0 = 0; h0 < NTO; h0 += NXH) {
        float tq[1][NXH][4], tk[1][NXH][4];
        acc_zero(tq);
        acc_zero(tk);
        for (int J = 0; J < nJ; ++J) {
          float pq[1][NXH][4], pk[1][NXH][4];
          acc_zero(pq);
          acc_zero(pk);
          warp_mma16_2a<NXH, true, false>(pq, pk, sDAqk + 16 * J, sDAkk + 16 * J, LDC, 16 * I,
                                          sKb + 16 * J * LDK, LDK, wc * DQ + 8 * h0, 16);
          const float* FIJ = sF + (I * (I + 1) / 2 + J) * D;
#pragma unroll
          for (int j = 0; j < NXH; ++j) {
            const float2 F2 = ld2<float>(FIJ + wc * DQ + 8 * (h0 + j) + 2 * tig);
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              setpr(tq[0][j], hf, fma2(F2, pr(pq[0][j], hf), pr(tq[0][j], hf)));
              setpr(tk[0][j], hf, fma2(F2, pr(pk[0][j], hf), pr(tk[0][j], hf)));
            }
          }
        }
#pragma unroll
        for (int j = 0; j < NXH; ++j)
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            const int jj = h0 + j;
            const int r = 16 * wr + gid + 8 * hf, c0 = wc * DQ + 8 * jj + 2 * tig;
            const float2 G2 = ld2<float>(sG + r * LDG + c0);
            const float2 Gb2 = ld2<float>(sG + (16 * I) * LDG + c0);
            const float2 q2 = ld2<T>(sq + r * LDK + c0), k2 = ld2<T>(sk + r * LDK + c0);
            const float2 b2 = ld2<T>(sb + r * LDK + c0);
            const float2 f = exp2_2(make_float2(G2.x - Gb2.x, G2.y - Gb2.y));
            const float2 xq = mul2(mul2(f2(scale), pr(tq[0][j], hf)), f);
            const float2 xk = mul2(pr(tk[0][j], hf), f);
            const float2 qn = mul2(q2, f2(rq[r]));
            const float2 kb = mul2(mul2(b2, k2), f2(rk[r]));
            setpr(dq[0][jj], hf, add2(pr(dq[0][jj], hf), xq));
            setpr(dkb[0][jj], hf, add2(pr(dkb[0][jj], hf), xk));
            setpr(dG[0][jj], hf, add2(pr(dG[0][jj], hf), fma2(qn, xq, mul2(kb, xk))));
          }
      }
    }
    // Y products: columns of block J = wr, from block rows I >= J; the key
    // side factor 2^(G_16I - G_r) = F_IJ 2^(G_(16J+15) - G_r)
    const int J = wr;
    constexpr int NYH = NTO >= 4 ? NTO / 2 : NTO;
#pragma unroll
    for (int h0 = 0; h0 < NTO; h0 += NYH) {
      float ys[NYH][4];
#pragma unroll
      for (int j = 0; j < NYH; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) ys[j][e] = 0.f;
      for (int I = J; I < 4; ++I) {
        if (I == J && !safe) continue;
        float ty[1][NYH][4];
        acc_zero(ty);
        warp_mma16<1, NYH, false, false>(ty, sDAqk + 16 * I * LDC, LDC, 16 * J,
                                         sQs + 16 * I * LDK, LDK, wc * DQ + 8 * h0, 16);
        warp_mma16<1, NYH, false, false>(ty, sDAkk + 16 * I * LDC, LDC, 16 * J,
                                         sKBs + 16 * I * LDK, LDK, wc * DQ + 8 * h0, 16);
        const float* FIJ = sF + (I * (I + 1) / 2 + J) * D;
#pragma unroll
        for (int j = 0; j < NYH; ++j) {
          const float2 F2 = ld2<float>(FIJ + wc * DQ + 8 * (h0 + j) + 2 * tig);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
            setpr(ys[j], hf, fma2(F2, pr(ty[0][j], hf), pr(ys[j], hf)));
        }
      }
#pragma unroll
      for (int j = 0; j < NYH; ++j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const int jj = h0 + j;
          const int r = 16 * wr + gid + 8 * hf, c0 = wc * DQ + 8 * jj + 2 * tig;
          const float2 Ge2 = ld2<float>(sG + (16 * J + 15) * LDG + c0);
          const float2 G2 = ld2<float>(sG + r * LDG + c0);
          const float2 k2 = ld2<T>(sk + r * LDK + c0);
          const float2 y = mul2(pr(ys[j], hf), exp2_2(make_float2(Ge2.x - G2.x, Ge2.y - G2.y)));
          const float2 kn = mul2(k2, f2(rk[r]));
          setpr(dkn[0][jj], hf, add2(pr(dkn[0][jj], hf), y));
          setpr(dG[0][jj], hf, fma2(neg2(kn), y, pr(dG[0][jj], hf)));
        }
    }
    if (!safe) {
      // exact diagonal block, off-diagonal pairs only
#pragma unroll
      for (int j = 0; j < NTO; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = 16 * wr + gid + ((e >> 1) << 3), cl = wc * DQ + 8 * j + 2 * tig + (e & 1);
          const float Gr = sG[r * LDG + cl];
          const float qn = to_f<T>(sq[r * LDK + cl]) * rq[r];
          const float kn = to_f<T>(sk[r * LDK + cl]) * rk[r];
          const float kb = to_f<T>(sb[r * LDK + cl]) * kn;
          float xq = 0.f, xk = 0.f, y = 0.f;
          for (int ii = 16 * wr; ii < 16 * wr + 16; ++ii) {
            if (ii < r) {
              const float ex = exp2f(Gr - sG[ii * LDG + cl]) * to_f<T>(sk[ii * LDK + cl]) * rk[ii];
              xq += scale * to_f<T>(sDAqk[r * LDC + ii]) * ex;
              xk += to_f<T>(sDAkk[r * LDC + ii]) * ex;
            } else if (ii > r) {
              const float ex = exp2f(sG[ii * LDG + cl] - Gr);
              const float qi = to_f<T>(sq[ii * LDK + cl]) * rq[ii];
              const float kbi = to_f<T>(sb[ii * LDK + cl]) * to_f<T>(sk[ii * LDK + cl]) * rk[ii];
              y += (scale * to_f<T>(sDAqk[ii * LDC + r]) * qi +
                    to_f<T>(sDAkk[ii * LDC + r]) * kbi) * ex;
            }
          }
          dq[0][j][e] += xq;
          dkb[0][j][e] += xk;
          dkn[0][j][e] += y;
          dG[0][j][e] += qn * xq + kb * xk - kn * y;
        }
    }
  }
  __syncthreads();  // score tiles are dead; W becomes the scan area

  // ---- dg = suffix scan of dG + prefix scan of the Kd terms -----------------
  float* sdG = reinterpret_cast<float*>(W + L::kdG);
  float* sX = TC ? sXs : reinterpret_cast<float*>(W + L::kX);
  float* sTmp = reinterpret_cast<float*>(W + L::kTmp);
#pragma unroll
  for (int j = 0; j < NTO; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf, c0 = wc * DQ + 8 * j + 2 * tig;
      float2 v = make_float2(dG[0][j][2 * hf], dG[0][j][2 * hf + 1]);
      if (r == len - 1) {
        v.x += dgl[c0] * exp2f(sG[(kChunk - 1) * LDG + c0]);
        v.y += dgl[c0 + 1] * exp2f(sG[(kChunk - 1) * LDG + c0 + 1]);
      }
      *reinterpret_cast<float2*>(sdG + r * LDG + c0) = v;
      if constexpr (!TC) {
        if (r + 1 < kChunk)
          *reinterpret_cast<float2*>(sX + (r + 1) * LDG + c0) =
              make_float2(X[j][2 * hf], X[j][2 * hf + 1]);
      }
    }
  for (int i = tid; i < D; i += NTH) sX[i] = 0.f;
  __syncthreads();
  // one register-staged pass: suffix sums of dG and prefix sums of the
  // shifted Kd terms down each column pair, added and stored straight to dg
  {
    constexpr int NC2 = D / 2, NSEG = NTH / NC2, RPS = kChunk / NSEG;
    static_assert(NSEG * NC2 == NTH && RPS * NSEG == kChunk, "scan shape");
    const int cp2 = tid % NC2, seg = tid / NC2, col = 2 * cp2;
    float2 su[RPS], px[RPS];
#pragma unroll
    for (int i = 0; i < RPS; ++i) {
      su[i] = ld2<float>(sdG + (seg * RPS + i) * LDG + col);
      px[i] = ld2<float>(sX + (seg * RPS + i) * LDG + col);
    }
#pragma unroll
    for (int i = 1; i < RPS; ++i) px[i] = add2(px[i], px[i - 1]);
#pragma unroll
    for (int i = RPS - 2; i >= 0; --i) su[i] = add2(su[i], su[i + 1]);
    float2* tP = reinterpret_cast<float2*>(sTmp);  // [NSEG][NC2] prefix, then suffix totals
    tP[seg * NC2 + cp2] = px[RPS - 1];
    tP[NTH + seg * NC2 + cp2] = su[0];
    __syncthreads();
    float2 offp = make_float2(0.f, 0.f), offs = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < NSEG; ++j) {
      if (j < seg) offp = add2(offp, tP[j * NC2 + cp2]);
      if (j > seg) offs = add2(offs, tP[NTH + j * NC2 + cp2]);
    }
    float* gdg = a.dg + offk;
    if (!a.gate.mode) {
#pragma unroll
      for (int i = 0; i < RPS; ++i) {
        const int r = seg * RPS + i;
        if (r < len && col < K)
          *reinterpret_cast<float2*>(gdg + (int64_t)r * ldk + col) =
              add2(add2(su[i], offs), add2(px[i], offp));
      }
    } else {
      // gate in kernel: dg of the raw input, plus this chunk's share of
      // dL/d dt_bias (per channel) and dL/dA_log (per head)
      const float* graw = a.g + offk;
      float sdt[2] = {0.f, 0.f}, sA = 0.f;
#pragma unroll
      for (int i = 0; i < RPS; ++i) {
        const int r = seg * RPS + i;
        if (r < len && col < K) {
          const float2 dyg = add2(add2(su[i], offs), add2(px[i], offp));
          float dA0, dA1;
          const float dg0 = gate_grad(a.gate, graw[(int64_t)r * ldk + col], dyg.x, h, col, K, &dA0);
          const float dg1 =
              gate_grad(a.gate, graw[(int64_t)r * ldk + col + 1], dyg.y, h, col + 1, K, &dA1);
          *reinterpret_cast<float2*>(gdg + (int64_t)r * ldk + col) = make_float2(dg0, dg1);
          sdt[0] += dg0;
          sdt[1] += dg1;
          sA += dA0 + dA1;
        }
      }
      if (a.gate.ddt_bias && col < K) {
        atomicAdd(a.gate.ddt_bias + h * K + col, sdt[0]);
        atomicAdd(a.gate.ddt_bias + h * K + col + 1, sdt[1]);
      }
      sA = warp_sum(sA);
      if (lane == 0) sDApart[warp] = sA;
    }
  }
  // (the staging tiles below reuse this area after the next barrier)

  // ---- db, dk, dq with the l2norm backward -------------------------------------
  T* gdq = reinterpret_cast<T*>(a.dq) + offk;
  T* gdk = reinterpret_cast<T*>(a.dk) + offk;
  T* gdb = reinterpret_cast<T*>(a.db) + offk;
  // staging tiles for coalesced stores (the scan area is dead after dg)
  T* stq = reinterpret_cast<T*>(W);
  T* stk = stq + kChunk * LDK;
  T* stb = stk + kChunk * LDK;
  // db is final here and goes to its staging tile at once; q and k stay
  // packed in registers for the l2norm pass
  float pq[2] = {0.f, 0.f}, pk[2] = {0.f, 0.f};
  uint32_t qpk[NTO][2], kpk[NTO][2];
#pragma unroll
  for (int j = 0; j < NTO; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf, c0 = wc * DQ + 8 * j + 2 * tig;
      qpk[j][hf] = *reinterpret_cast<const uint32_t*>(sq + r * LDK + c0);
      kpk[j][hf] = *reinterpret_cast<const uint32_t*>(sk + r * LDK + c0);
      const float2 q2 = unpack2<T>(qpk[j][hf]), k2 = unpack2<T>(kpk[j][hf]);
      const float2 b2 = ld2<T>(sb + r * LDK + c0);
      const float2 dgn = f2(scale * sDiag[r]);
      const float2 qn = mul2(q2, f2(rq[r])), kn = mul2(k2, f2(rk[r]));
      const float2 dkbv = pr(dkb[0][j], hf);
      const float2 dqv = fma2(dgn, kn, pr(dq[0][j], hf));
      const float2 dknv = add2(pr(dkn[0][j], hf), fma2(dkbv, b2, mul2(dgn, qn)));
      setpr(dq[0][j], hf, dqv);
      setpr(dkn[0][j], hf, dknv);
      const float2 db2 = mul2(dkbv, kn);
      *reinterpret_cast<uint32_t*>(stb + r * LDK + c0) = pack2<T>(db2.x, db2.y);
      pq[hf] = fmaf(qn.y, dqv.y, fmaf(qn.x, dqv.x, pq[hf]));
      pk[hf] = fmaf(kn.y, dknv.y, fmaf(kn.x, dknv.x, pk[hf]));
    }
  if (a.l2norm) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      pq[hf] += __shfl_xor_sync(0xffffffffu, pq[hf], 1);
      pq[hf] += __shfl_xor_sync(0xffffffffu, pq[hf], 2);
      pk[hf] += __shfl_xor_sync(0xffffffffu, pk[hf], 1);
      pk[hf] += __shfl_xor_sync(0xffffffffu, pk[hf], 2);
    }
    if (tig == 0) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        pdq[wc * 64 + 16 * wr + gid + 8 * hf] = pq[hf];
        pdk[wc * 64 + 16 * wr + gid + 8 * hf] = pk[hf];
      }
    }
  }
  __syncthreads();
  if (a.gate.mode && tid == 0 && a.gate.dA_log) {
    float sA = 0.f;
    for (int i = 0; i < NTH / 32; ++i) sA += sDApart[i];
    atomicAdd(a.gate.dA_log + h, sA);
  }
  float dotq[2] = {0.f, 0.f}, dotk[2] = {0.f, 0.f};
  if (a.l2norm) {
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf;
      dotq[hf] = pdq[r] + pdq[64 + r] + pdq[128 + r] + pdq[192 + r];
      dotk[hf] = pdk[r] + pdk[64 + r] + pdk[128 + r] + pdk[192 + r];
    }
  }
#pragma unroll
  for (int j = 0; j < NTO; ++j)
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
      const int r = 16 * wr + gid + 8 * hf, cl = wc * DQ + 8 * j + 2 * tig;
      if (r >= len || cl >= K) continue;
      float2 oq = pr(dq[0][j], hf), ok = pr(dkn[0][j], hf);
      if (a.l2norm) {
        const float2 q2 = unpack2<T>(qpk[j][hf]), k2 = unpack2<T>(kpk[j][hf]);
        const float2 nq = f2(rq[r]), nk = f2(rk[r]);
        oq = mul2(fma2(neg2(mul2(q2, nq)), f2(dotq[hf]), oq), nq);
        ok = mul2(fma2(neg2(mul2(k2, nk)), f2(dotk[hf]), ok), nk);
      }
      *reinterpret_cast<uint32_t*>(stq + r * LDK + cl) = pack2<T>(oq.x, oq.y);
      *reinterpret_cast<uint32_t*>(stk + r * LDK + cl) = pack2<T>(ok.x, ok.y);
    }
  __syncthreads();
  store_tile16<T, kChunk, D, NTH>(gdq, ldk, stq, LDK, len, K);
  store_tile16<T, kChunk, D, NTH>(gdk, ldk, stk, LDK, len, K);
  store_tile16<T, kChunk, D, NTH>(gdb, ldk, stb, LDK, len, K);
  if constexpr (TC) {
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
      tc::tc_fence_after();
      tc::tmem_dealloc(tmem, 256);
    }
  }
}

// K = V = 128 takes the tcgen05 value phase: h / dh as [128][64] and dO, v,
// w, VN^T, dVN^T as [64][64] boxes of 128-byte-swizzled tiles; A, q, k, b, g
// keep their padded unswizzled boxes.
template <typename T>
cudaError_t launch_bwd_intra16_tc(const BwdIntraArgs& a, cudaStream_t st) {
  using L = Bwd16Layout<128, true>;
  auto kern = k_bwd_intra16<T, 128, true>;
  const uint64_t nch = (uint64_t)a.seqs.n_chunks, H = (uint64_t)a.H, rows = (uint64_t)a.total_rows;
  constexpr uint64_t K = 128, V = 128;
  Bwd16Maps m;
  const uint64_t dK[3] = {K, H, rows}, sK[2] = {K * 2, H * K * 2}, sG[2] = {K * 4, H * K * 4};
  const uint32_t bK[3] = {(uint32_t)L::LDK, 1, kChunk}, bG[3] = {(uint32_t)L::LDG, 1, kChunk};
  const uint64_t dA[2] = {kChunk, nch * H * kChunk}, s64[1] = {kChunk * 2};
  const uint32_t bA[2] = {(uint32_t)L::LDC, kChunk};
  const unsigned char* sv = a.saved;
  const unsigned char* wv = a.ws;
  if (!tmap_plain(&m.q, a.q, 3, dK, sK, bK, 2) || !tmap_plain(&m.k, a.k, 3, dK, sK, bK, 2) ||
      !tmap_plain(&m.b, a.b, 3, dK, sK, bK, 2) || !tmap_plain(&m.g, a.g, 3, dK, sG, bG, 4) ||
      !tmap_plain(&m.a, sv + a.L.a, 2, dA, s64, bA, 2) ||
      !tmap_rows(&m.dout, a.dout, V, H, rows, 64, 2) || !tmap_rows(&m.v, a.v, V, H, rows, 64, 2) ||
      !tmap_rows(&m.w, a.w, V, H, rows, 64, 2) ||
      !tmap_2d_box_bf16(&m.h, sv + a.L.h, V, nch * H * K, 64, 128) ||
      !tmap_2d_box_bf16(&m.dh, wv + a.BL.dh, V, nch * H * K, 64, 128) ||
      !tmap_2d_bf16(&m.vn, sv + a.L.vn, kChunk, nch * H * V, 64, true) ||
      !tmap_2d_bf16(&m.dvn, wv + a.BL.dvn, kChunk, nch * H * V, 64, true))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)L::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(a.seqs.n_chunks, a.H);
  kern<<<grid, kThreadsB16, L::bytes, st>>>(a, m);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_bwd_intra16(const BwdIntraArgs& a, cudaStream_t st) {
  using L = Bwd16Layout<D>;
  auto kern = k_bwd_intra16<T, D, false>;
  const uint64_t nch = (uint64_t)a.seqs.n_chunks, H = (uint64_t)a.H, K = (uint64_t)a.K,
                 V = (uint64_t)a.V, rows = (uint64_t)a.total_rows;
  if (nch == 0 || H == 0) return cudaSuccess;
  // TMA coordinates are 32-bit
  const uint64_t lim = (uint64_t)1 << 31;
  if (rows >= lim || nch * H * (K > V ? K : V) >= lim || nch * H * kChunk >= lim)
    return cudaErrorInvalidValue;
  if constexpr (D == 128) {
    if (K == 128 && V == 128 && tmap_available()) return launch_bwd_intra16_tc<T>(a, st);
  }
  Bwd16Maps m;
  const uint64_t dK[3] = {K, H, rows}, sK[2] = {K * 2, H * K * 2}, sG[2] = {K * 4, H * K * 4};
  const uint64_t dV[3] = {V, H, rows}, sV[2] = {V * 2, H * V * 2};
  const uint32_t bK[3] = {(uint32_t)L::LDK, 1, kChunk}, bG[3] = {(uint32_t)L::LDG, 1, kChunk};
  const uint32_t bV[3] = {(uint32_t)L::LDS, 1, kChunk};
  const uint64_t dH[2] = {V, nch * H * K}, sH[1] = {V * 2};
  const uint32_t bH[2] = {(uint32_t)L::LDS, (uint32_t)K};
  const uint64_t dVN[2] = {kChunk, nch * H * V}, dA[2] = {kChunk, nch * H * kChunk};
  const uint64_t s64[1] = {kChunk * 2};
  const uint32_t bVN[2] = {(uint32_t)L::LDT, 32}, bA[2] = {(uint32_t)L::LDC, kChunk};
  const unsigned char* sv = a.saved;
  const unsigned char* wv = a.ws;
  if (!tmap_plain(&m.q, a.q, 3, dK, sK, bK, 2) || !tmap_plain(&m.k, a.k, 3, dK, sK, bK, 2) ||
      !tmap_plain(&m.b, a.b, 3, dK, sK, bK, 2) || !tmap_plain(&m.g, a.g, 3, dK, sG, bG, 4) ||
      !tmap_plain(&m.dout, a.dout, 3, dV, sV, bV, 2) || !tmap_plain(&m.v, a.v, 3, dV, sV, bV, 2) ||
      !tmap_plain(&m.w, a.w, 3, dV, sV, bV, 2) ||
      !tmap_plain(&m.h, sv + a.L.h, 2, dH, sH, bH, 2) ||
      !tmap_plain(&m.dh, wv + a.BL.dh, 2, dH, sH, bH, 2) ||
      !tmap_plain(&m.vn, sv + a.L.vn, 2, dVN, s64, bVN, 2) ||
      !tmap_plain(&m.dvn, wv + a.BL.dvn, 2, dVN, s64, bVN, 2) ||
      !tmap_plain(&m.a, sv + a.L.a, 2, dA, s64, bA, 2))
    return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)L::bytes);
  if (e != cudaSuccess) return e;
  dim3 grid(a.seqs.n_chunks, a.H);
  kern<<<grid, kThreadsB16, L::bytes, st>>>(a, m);
  return cudaGetLastError();
}
template cudaError_t launch_bwd_intra16<__nv_bfloat16, 64>(const BwdIntraArgs&, cudaStream_t);
template cudaError_t launch_bwd_intra16<__nv_bfloat16, 128>(const BwdIntraArgs&, cudaStream_t);

}  // namespace gdn2
