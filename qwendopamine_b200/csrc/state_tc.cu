// state_tc.cu -- forward inter-chunk state pass on the 5th-generation tensor
// cores (tcgen05 + TMEM + TMA), bf16 inputs, K = V = 128.
//
// One CTA of 8 warps per (sequence, head) walks the sequence's chunks in
// order.  Tensor memory (256 columns x 128 lanes, fp32) holds
//   cols [0,128)   the state h           (lane = key row k, column = value v)
//   cols [128,192) VN^T = h^T W^T, then U^T - that  (lane = v, column = token)
//   cols [192,256) o^T = h^T Qg^T + VN^T Aqk^T      (lane = v, column = token)
// so the state never leaves the SM between chunks.  Per chunk:
//   1. one thread issues  VN^T = h^T W^T  and  o^T = h^T Qg^T  (A = bf16 h in
//      shared memory, MN-major; B = W / Qg tiles, K-major), commits; the
//      other threads meanwhile copy the chunk's checkpoint and the previous
//      chunk's o out of their shared-memory staging tiles;
//   2. all warps read VN^T, form VN = U - W h and write bf16 VN^T (K-major)
//      to shared memory;
//   3. one thread issues  o^T += VN^T Aqk^T  and  h += Kd^T VN  (A = Kd tile,
//      MN-major; B = VN^T, K-major) onto the state already scaled by 2^G_last;
//      meanwhile VN^T is copied to the saved buffer;
//   4. all warps stage o, read the new state, write its bf16 copy (operand of
//      the next chunk and its checkpoint) and scale it in place by the next
//      chunk's 2^G_last.
// Every global store is a 16-byte vector and each warp instruction writes
// 512 contiguous bytes (a transposing store from TMEM lanes would scatter).
// The per-chunk tiles (W, Qg, Kd, Aqk: 128-byte swizzled; U: plain; gl: bulk)
// arrive by TMA into a two-slot ring, two chunks ahead.  Every wait on an
// mbarrier is bounded in time; a wait that runs out marks the CTA aborted,
// all warps leave the chunk loop together, in-flight copies are waited for
// (bounded), the tensor memory is freed and a fault bit is set in
// g_gdn2_fault for gdn2_fault_status() to report.
//
// Same recurrence and rounding points as k_fwd_state16 (state16.cu): fp32
// state, bf16 copies of h and VN as product operands, fp32 accumulation.
#include <cuda.h>

#include "chunk_args.cuh"
#include "tc.cuh"

namespace gdn2 {

__device__ unsigned int g_gdn2_fault;

namespace {

constexpr int kTcThreads = 256;
constexpr uint32_t kBox = 8192;  // one 64-row x 128-byte TMA box
// per-chunk slot (bytes, 1024-aligned pieces)
constexpr uint32_t kOffW = 0;
constexpr uint32_t kOffQg = 2 * kBox;
constexpr uint32_t kOffKd = 4 * kBox;
constexpr uint32_t kOffAqk = 6 * kBox;
constexpr uint32_t kOffU = 7 * kBox;  // [64][128] bf16, unswizzled
constexpr uint32_t kOffGl = 9 * kBox; // [128] fp32
constexpr uint32_t kGlBytes = 128 * 4;
constexpr uint32_t kSlotBytes = 9 * kBox + 1024;
constexpr uint32_t kTxBytes = 9 * kBox + kGlBytes;
// persistent operands and staging
constexpr uint32_t kOffH = 2 * kSlotBytes;     // bf16 h [k][v], MN-major SW128 (32 KB)
constexpr uint32_t kHalfH = 2 * kBox;          // v-halves of it are 16 KB apart
constexpr uint32_t kOffVN = kOffH + 4 * kBox;  // bf16 VN^T [v][t], K-major SW128 (16 KB)
constexpr uint32_t kOffO = kOffVN + 2 * kBox;  // bf16 o [t][v], row-major (16 KB)
constexpr uint32_t kOffBar = kOffO + 2 * kBox;
constexpr uint32_t kSmemBytes = kOffBar + 64 + 1024;  // + alignment slack

constexpr uint32_t kColH = 0, kColVN = 128, kColO = 192, kTmemCols = 256;

// instruction descriptors
constexpr uint32_t kIdHW = tc::idesc_bf16(128, 64, 1, 0);    // h^T W^T, h^T Qg^T
constexpr uint32_t kIdVA = tc::idesc_bf16(128, 64, 0, 0);    // VN^T Aqk^T
constexpr uint32_t kIdKV = tc::idesc_bf16(128, 128, 1, 0);   // Kd^T VN

// Operand descriptors from shared-memory addresses in 16-byte units (tile
// bases are 1024-byte aligned, so every offset below is a whole unit).
__device__ __forceinline__ uint64_t desc_k(uint32_t a16) {  // K-major, 128B swizzle
  return tc::sdesc_layout(16, 1024, tc::kSwizzle128) | a16;
}
__device__ __forceinline__ uint64_t desc_mn(uint32_t a16, uint32_t mn_stride) {  // MN-major
  return tc::sdesc_layout(mn_stride, 1024, tc::kSwizzle128) | a16;
}

__device__ __forceinline__ void st_shared_v4(void* p, uint4 x) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(smem_u32(p)), "r"(x.x), "r"(x.y),
               "r"(x.z), "r"(x.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_shared_v4(const void* p) {
  uint4 x;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(x.x), "=r"(x.y), "=r"(x.z), "=r"(x.w)
               : "r"(smem_u32(p)));
  return x;
}

__global__ void __launch_bounds__(kTcThreads, 1)
    k_fwd_state_tc(FwdStateArgs a, const __grid_constant__ CUtensorMap mW,
                   const __grid_constant__ CUtensorMap mQg, const __grid_constant__ CUtensorMap mKd,
                   const __grid_constant__ CUtensorMap mAqk, const __grid_constant__ CUtensorMap mU) {
  using T = __nv_bfloat16;
  constexpr int K = 128, V = 128;
  extern __shared__ unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);  // [2]
  uint64_t* mma1 = full + 2;
  uint64_t* mma2 = full + 3;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
  unsigned char* sH = sm + kOffH;
  const uint32_t sH16 = (smem_u32(sm) >> 4) + (kOffH >> 4);
  unsigned char* sVN = sm + kOffVN;
  const uint32_t sVN16 = (smem_u32(sm) >> 4) + (kOffVN >> 4);
  unsigned char* sO = sm + kOffO;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;  // the TMEM lane this thread reads
  const int H = a.H;
  const int nh = blockIdx.x, n = nh / H, h = nh - n * H;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];
  const int64_t bos = a.seqs.cu[n], eos = a.seqs.cu[n + 1];
  const int64_t ldo = (int64_t)H * V;
  const float* h0 = a.h0 ? a.h0 + (int64_t)nh * K * V : nullptr;
  float* ht = a.ht ? a.ht + (int64_t)nh * K * V : nullptr;
  const uint64_t lim = a.wait_ns ? a.wait_ns : tc::kWaitLimitNs;

  if (c_begin >= c_end) {  // empty sequence: the state passes through
    if (ht)
      for (int i = tid; i < K * V; i += kTcThreads) ht[i] = h0 ? h0[i] : 0.f;
    return;
  }

  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(mma1, 1);
    tc::mbar_init(mma2, 1);
    *sAbort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(sTmem, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *sTmem;
  const uint32_t tlane = tmem + ((uint32_t)(quad * 32) << 16);

  // ---- producer (thread 0) --------------------------------------------------
  int next_issue = c_begin;  // meaningful in thread 0 only
  int mma1_commits = 0, mma2_commits = 0;
  auto issue = [&](int c) {
    if (c == a.skip_chunk) {  // test of the abort path: this chunk never arrives
      next_issue = c + 1;
      return;
    }
    const int slot = (c - c_begin) & 1;
    unsigned char* p = sm + slot * kSlotBytes;
    const size_t ch = (size_t)c * H + h;
    const int y = (int)(ch * kChunk);
    tc::mbar_expect_tx(&full[slot], kTxBytes);
    tc::tma_load_2d(p + kOffW, &mW, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffW + kBox, &mW, 64, y, &full[slot]);
    tc::tma_load_2d(p + kOffQg, &mQg, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffQg + kBox, &mQg, 64, y, &full[slot]);
    tc::tma_load_2d(p + kOffKd, &mKd, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffKd + kBox, &mKd, 64, y, &full[slot]);
    tc::tma_load_2d(p + kOffAqk, &mAqk, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffU, &mU, 0, y, &full[slot]);
    tc::bulk_load(p + kOffGl, a.saved + a.L.gl + ch * K * sizeof(float), kGlBytes, &full[slot]);
    next_issue = c + 1;
  };
  if (tid == 0) {
    issue(c_begin);
    if (c_begin + 1 < c_end) issue(c_begin + 1);
  }

  // bf16 copy of this thread's 64 state values (row k = `row`, columns
  // 64*half ..) into the MN-major operand tile.
  auto emit_state = [&](const float (&s)[64]) {
    unsigned char* srow = sH + half * kHalfH + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint4 x;
      x.x = pack2<T>(s[8 * q + 0], s[8 * q + 1]);
      x.y = pack2<T>(s[8 * q + 2], s[8 * q + 3]);
      x.z = pack2<T>(s[8 * q + 4], s[8 * q + 5]);
      x.w = pack2<T>(s[8 * q + 6], s[8 * q + 7]);
      st_shared_v4(srow + ((q ^ (row & 7)) << 4), x);
    }
  };
  auto scale_store = [&](float (&s)[64], int slot) {
    const float gl = reinterpret_cast<const float*>(sm + slot * kSlotBytes + kOffGl)[row];
    float lo[32], hi[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      lo[i] = s[i] * gl;
      hi[i] = s[32 + i] * gl;
    }
    tc::tmem_st32(tlane + kColH + 64 * half, lo);
    tc::tmem_st32(tlane + kColH + 64 * half + 32, hi);
  };
  // Coalesced copies out of the staging tiles (all 256 threads; each warp
  // instruction moves 512 contiguous bytes).
  auto copy_ckpt = [&](int c) {  // sH -> checkpoint of chunk c, [K][V]
    T* gh = reinterpret_cast<T*>(a.saved + a.L.h) + ((size_t)c * H + h) * (size_t)K * V;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int idx = tid + it * kTcThreads;
      const int k = idx >> 4, ci = idx & 15;
      const uint4 x = ld_shared_v4(sH + (ci >> 3) * kHalfH + (k >> 3) * 1024 + (k & 7) * 128 +
                                   (((ci & 7) ^ (k & 7)) << 4));
      *reinterpret_cast<uint4*>(gh + (size_t)k * V + 8 * ci) = x;
    }
  };
  auto copy_vn = [&](int c) {  // sVN -> VN^T of chunk c, [V][64]
    T* gv = reinterpret_cast<T*>(a.saved + a.L.vn) + ((size_t)c * H + h) * (size_t)kChunk * V;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = tid + it * kTcThreads;
      const int v = idx >> 3, ci = idx & 7;
      const uint4 x = ld_shared_v4(sVN + (v >> 3) * 1024 + (v & 7) * 128 + ((ci ^ (v & 7)) << 4));
      *reinterpret_cast<uint4*>(gv + (size_t)v * kChunk + 8 * ci) = x;
    }
  };
  auto copy_o = [&](int c) {  // sO -> output rows of chunk c
    const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);
    T* go = reinterpret_cast<T*>(a.o) + cp.row0 * ldo + (int64_t)h * V;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = tid + it * kTcThreads;
      const int t = idx >> 4, ci = idx & 15;
      if (t < cp.len)
        *reinterpret_cast<uint4*>(go + (int64_t)t * ldo + 8 * ci) =
            ld_shared_v4(sO + t * (V * 2) + ci * 16);
    }
  };

  // ---- initial state ----------------------------------------------------------
  {
    const bool ok = tc::warp_wait(&full[0], 0, lim);
    if (ok) {
      float s[64];
      if (h0) {
        const float4* src = reinterpret_cast<const float4*>(h0 + (size_t)row * V + 64 * half);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 x = src[i];
          s[4 * i] = x.x;
          s[4 * i + 1] = x.y;
          s[4 * i + 2] = x.z;
          s[4 * i + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = 0.f;
      }
      emit_state(s);
      scale_store(s, 0);
    } else if (lane == 0) {
      *sAbort = 1;
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
  }

  int c = c_begin;
  if (!*sAbort) {
    for (; c < c_end; ++c) {
      const int i = c - c_begin, slot = i & 1;
      unsigned char* p = sm + slot * kSlotBytes;
      const uint32_t p16 = (smem_u32(sm) >> 4) + slot * (kSlotBytes >> 4);
      const uint32_t par_full = (i >> 1) & 1, par_mma = i & 1;

      // 1. VN^T = h^T W^T,  o^T = h^T Qg^T;  meanwhile the checkpoint of
      //    chunk c and the previous chunk's o leave through the copy units.
      if (tid == 0) {
        if (!tc::mbar_wait(&full[slot], par_full, lim)) {
          *sAbort = 1;
        } else {
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::umma_bf16(tmem + kColVN, desc_mn(sH16 + ((j * 2048) >> 4), kHalfH),
                          desc_k(p16 + ((kOffW + (j >> 2) * kBox + (j & 3) * 32) >> 4)), kIdHW, j > 0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::umma_bf16(tmem + kColO, desc_mn(sH16 + ((j * 2048) >> 4), kHalfH),
                          desc_k(p16 + ((kOffQg + (j >> 2) * kBox + (j & 3) * 32) >> 4)), kIdHW, j > 0);
          tc::umma_commit(mma1);
          ++mma1_commits;
        }
      }
      copy_ckpt(c);
      if (c > c_begin) copy_o(c - 1);
      // 2. VN = U - W h  -> bf16 VN^T operand tile
      {
        bool ok = tc::warp_wait(mma1, par_mma, lim);
        if (ok) ok = tc::warp_wait(&full[slot], par_full, lim);
        if (ok) {
          tc::tc_fence_after();
          uint32_t x[32];
          tc::tmem_ld32(tlane + kColVN + 32 * half, x);
          const T* sU = reinterpret_cast<const T*>(p + kOffU) + row;
          float u[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) u[e] = to_f<T>(sU[(32 * half + e) * V]);
          tc::tmem_wait_ld();
          unsigned char* vrow = sVN + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 y;
            y.x = pack2<T>(u[8 * q + 0] - __uint_as_float(x[8 * q + 0]),
                           u[8 * q + 1] - __uint_as_float(x[8 * q + 1]));
            y.y = pack2<T>(u[8 * q + 2] - __uint_as_float(x[8 * q + 2]),
                           u[8 * q + 3] - __uint_as_float(x[8 * q + 3]));
            y.z = pack2<T>(u[8 * q + 4] - __uint_as_float(x[8 * q + 4]),
                           u[8 * q + 5] - __uint_as_float(x[8 * q + 5]));
            y.w = pack2<T>(u[8 * q + 6] - __uint_as_float(x[8 * q + 6]),
                           u[8 * q + 7] - __uint_as_float(x[8 * q + 7]));
            st_shared_v4(vrow + (((4 * half + q) ^ (row & 7)) << 4), y);
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      // 3. o^T += VN^T Aqk^T,  h += Kd^T VN;  meanwhile VN^T leaves.
      if (tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kColO, desc_k(sVN16 + ((j * 32) >> 4)), desc_k(p16 + ((kOffAqk + j * 32) >> 4)), kIdVA, 1);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kColH, desc_mn(p16 + ((kOffKd + j * 2048) >> 4), kBox), desc_k(sVN16 + ((j * 32) >> 4)),
                        kIdKV, 1);
        tc::umma_commit(mma2);
        ++mma2_commits;
      }
      copy_vn(c);
      // 4. o -> staging; new state -> bf16 operand tile (the next checkpoint),
      //    scaled in place by the next chunk's 2^G_last
      {
        const bool has_next = c + 1 < c_end;
        bool ok = tc::warp_wait(mma2, par_mma, lim);
        if (ok && has_next) ok = tc::warp_wait(&full[slot ^ 1], ((i + 1) >> 1) & 1, lim);
        if (ok) {
          tc::tc_fence_after();
          {
            uint32_t x[32];
            tc::tmem_ld32(tlane + kColO + 32 * half, x);
            tc::tmem_wait_ld();
            T* orow = reinterpret_cast<T*>(sO) + row;
#pragma unroll
            for (int e = 0; e < 32; ++e) orow[(32 * half + e) * V] = from_f<T>(__uint_as_float(x[e]));
          }
          float s[64];
          {
            uint32_t lo[32], hi[32];
            tc::tmem_ld32(tlane + kColH + 64 * half, lo);
            tc::tmem_ld32(tlane + kColH + 64 * half + 32, hi);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              s[e] = __uint_as_float(lo[e]);
              s[32 + e] = __uint_as_float(hi[e]);
            }
          }
          if (has_next) {
            emit_state(s);
            scale_store(s, slot ^ 1);
          } else if (ht) {
            float4* dst = reinterpret_cast<float4*>(ht + (size_t)row * V + 64 * half);
#pragma unroll
            for (int e = 0; e < 16; ++e)
              dst[e] = make_float4(s[4 * e], s[4 * e + 1], s[4 * e + 2], s[4 * e + 3]);
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      if (tid == 0 && c + 2 < c_end) issue(c + 2);
    }
  }

  // ---- teardown ---------------------------------------------------------------
  const bool aborted = *sAbort != 0;
  if (!aborted) copy_o(c_end - 1);
  if (aborted && tid == 0) {
    // let copies and products already in flight finish before the shared
    // and tensor memory they target is released (each wait bounded)
    for (int j = c; j < next_issue; ++j) {
      const int ij = j - c_begin;
      tc::mbar_wait(&full[ij & 1], (ij >> 1) & 1, lim);
    }
    if (mma1_commits > 0) tc::mbar_wait(mma1, (mma1_commits - 1) & 1, lim);
    if (mma2_commits > 0) tc::mbar_wait(mma2, (mma2_commits - 1) & 1, lim);
    atomicOr(&g_gdn2_fault, 1u);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Backward state pass, reverse over the chunks of one (sequence, head):
//   dVN = Aqk^T dO + Kd dh,   dh <- gl * dh + Qg^T dO - W^T dVN
// TMEM: cols [0,128) dh (lane = key row k), cols [128,192) dVN^T (lane = v).
// dO arrives by TMA through a 3-D view [rows][H][V] (rows of a partial chunk
// past the sequence's end are zeroed in shared memory before use).  Per
// chunk: checkpoint dh (bf16, the gradient of the state leaving the chunk)
// while  dVN^T = dO^T Aqk + dh^T Kd^T  runs (A = dO tile, MN-major; B = Aqk,
// MN-major / A = bf16 dh, MN-major; B = Kd, K-major); warps store -dVN^T
// (K-major) for  dh += Qg^T dO + W^T (-dVN)  (A = Qg / W tiles, MN-major;
// B = dO, MN-major / -dVN^T, K-major) and copy dVN^T out while it runs; then
// the new dh becomes the next operand, scaled in TMEM by the next chunk's
// 2^G_last.  Same rounding points as k_bwd_state16.
constexpr uint32_t kOffDO = kOffU;  // dO takes U's place: 2 swizzled boxes
constexpr uint32_t kIdOA = tc::idesc_bf16(128, 64, 1, 1);   // dO^T Aqk
constexpr uint32_t kIdQO = tc::idesc_bf16(128, 128, 1, 1);  // Qg^T dO

__global__ void __launch_bounds__(kTcThreads, 1)
    k_bwd_state_tc(BwdStateArgs a, const __grid_constant__ CUtensorMap mW,
                   const __grid_constant__ CUtensorMap mQg, const __grid_constant__ CUtensorMap mKd,
                   const __grid_constant__ CUtensorMap mAqk, const __grid_constant__ CUtensorMap mDO) {
  using T = __nv_bfloat16;
  constexpr int K = 128, V = 128;
  extern __shared__ unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);  // [2]
  uint64_t* mma1 = full + 2;
  uint64_t* mma2 = full + 3;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
  unsigned char* sH = sm + kOffH;    // bf16 dh [k][v], MN-major
  const uint32_t sH16 = (smem_u32(sm) >> 4) + (kOffH >> 4);
  unsigned char* sVN = sm + kOffVN;  // bf16 -dVN^T [v][t], K-major
  const uint32_t sVN16 = (smem_u32(sm) >> 4) + (kOffVN >> 4);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;
  const int H = a.H;
  const int nh = blockIdx.x, n = nh / H, h = nh - n * H;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];
  const int64_t bos = a.seqs.cu[n], eos = a.seqs.cu[n + 1];
  const float* dht = a.dht ? a.dht + (int64_t)nh * K * V : nullptr;
  float* dh0 = a.dh0 ? a.dh0 + (int64_t)nh * K * V : nullptr;

  if (c_begin >= c_end) {  // empty sequence: the gradient passes through
    if (dh0)
      for (int i = tid; i < K * V; i += kTcThreads) dh0[i] = dht ? dht[i] : 0.f;
    return;
  }

  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(mma1, 1);
    tc::mbar_init(mma2, 1);
    *sAbort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(sTmem, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *sTmem;
  const uint32_t tlane = tmem + ((uint32_t)(quad * 32) << 16);

  // chunk c sits in slot (c_end - 1 - c) & 1
  int next_issue = c_end - 1;  // next chunk to request (thread 0), counting down
  int mma1_commits = 0, mma2_commits = 0;
  auto issue = [&](int c) {
    const int slot = (c_end - 1 - c) & 1;
    unsigned char* p = sm + slot * kSlotBytes;
    const size_t ch = (size_t)c * H + h;
    const int y = (int)(ch * kChunk);
    const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);
    tc::mbar_expect_tx(&full[slot], kTxBytes);
    tc::tma_load_2d(p + kOffW, &mW, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffW + kBox, &mW, 64, y, &full[slot]);
    tc::tma_load_2d(p + kOffQg, &mQg, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffQg + kBox, &mQg, 64, y, &full[slot]);
    tc::tma_load_2d(p + kOffKd, &mKd, 0, y, &full[slot]);
    tc::tma_load_2d(p + kOffKd + kBox, &mKd, 64, y, &full[slot]);
    tc::tma_load_2d(p + kOffAqk, &mAqk, 0, y, &full[slot]);
    tc::tma_load_3d(p + kOffDO, &mDO, 0, h, (int)cp.row0, &full[slot]);
    tc::tma_load_3d(p + kOffDO + kBox, &mDO, 64, h, (int)cp.row0, &full[slot]);
    tc::bulk_load(p + kOffGl, a.saved + a.L.gl + ch * K * sizeof(float), kGlBytes, &full[slot]);
    next_issue = c - 1;
  };
  if (tid == 0) {
    issue(c_end - 1);
    if (c_end - 2 >= c_begin) issue(c_end - 2);
  }

  auto emit_state = [&](const float (&s)[64]) {
    unsigned char* srow = sH + half * kHalfH + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      uint4 x;
      x.x = pack2<T>(s[8 * q + 0], s[8 * q + 1]);
      x.y = pack2<T>(s[8 * q + 2], s[8 * q + 3]);
      x.z = pack2<T>(s[8 * q + 4], s[8 * q + 5]);
      x.w = pack2<T>(s[8 * q + 6], s[8 * q + 7]);
      st_shared_v4(srow + ((q ^ (row & 7)) << 4), x);
    }
  };
  auto scale_store = [&](float (&s)[64], int slot) {
    const float gl = reinterpret_cast<const float*>(sm + slot * kSlotBytes + kOffGl)[row];
    float lo[32], hi[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      lo[i] = s[i] * gl;
      hi[i] = s[32 + i] * gl;
    }
    tc::tmem_st32(tlane + kColH + 64 * half, lo);
    tc::tmem_st32(tlane + kColH + 64 * half + 32, hi);
  };
  auto copy_ckpt = [&](int c) {  // sH -> dh of chunk c, [K][V]
    T* gh = reinterpret_cast<T*>(a.ws + a.BL.dh) + ((size_t)c * H + h) * (size_t)K * V;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int idx = tid + it * kTcThreads;
      const int k = idx >> 4, ci = idx & 15;
      const uint4 x = ld_shared_v4(sH + (ci >> 3) * kHalfH + (k >> 3) * 1024 + (k & 7) * 128 +
                                   (((ci & 7) ^ (k & 7)) << 4));
      *reinterpret_cast<uint4*>(gh + (size_t)k * V + 8 * ci) = x;
    }
  };
  auto copy_dvn = [&](int c) {  // -sVN -> dVN^T of chunk c, [V][64]
    T* gv = reinterpret_cast<T*>(a.ws + a.BL.dvn) + ((size_t)c * H + h) * (size_t)kChunk * V;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = tid + it * kTcThreads;
      const int v = idx >> 3, ci = idx & 7;
      uint4 x = ld_shared_v4(sVN + (v >> 3) * 1024 + (v & 7) * 128 + ((ci ^ (v & 7)) << 4));
      x.x ^= 0x80008000u;  // flip the bf16 signs back
      x.y ^= 0x80008000u;
      x.z ^= 0x80008000u;
      x.w ^= 0x80008000u;
      *reinterpret_cast<uint4*>(gv + (size_t)v * kChunk + 8 * ci) = x;
    }
  };

  // ---- initial gradient -----------------------------------------------------
  {
    const bool ok = tc::warp_wait(&full[0], 0);
    if (ok) {
      float s[64];
      if (dht) {
        const float4* src = reinterpret_cast<const float4*>(dht + (size_t)row * V + 64 * half);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 x = src[i];
          s[4 * i] = x.x;
          s[4 * i + 1] = x.y;
          s[4 * i + 2] = x.z;
          s[4 * i + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = 0.f;
      }
      emit_state(s);
      scale_store(s, 0);
    } else if (lane == 0) {
      *sAbort = 1;
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
  }

  int c = c_end - 1;
  if (!*sAbort) {
    for (; c >= c_begin; --c) {
      const int i = c_end - 1 - c, slot = i & 1;
      unsigned char* p = sm + slot * kSlotBytes;
      const uint32_t p16 = (smem_u32(sm) >> 4) + slot * (kSlotBytes >> 4);
      const uint32_t par_full = (i >> 1) & 1, par_mma = i & 1;
      const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);

      // 0. a partial chunk's dO rows past the sequence end hold the next
      //    sequence's tokens: zero them before any product reads the tile
      if (cp.len < kChunk) {
        const bool ok = tc::warp_wait(&full[slot], par_full);
        if (ok) {
          for (int e = tid; e < (kChunk - cp.len) * 16; e += kTcThreads) {
            const int r = cp.len + (e >> 4), bx = (e >> 3) & 1, ci = e & 7;
            st_shared_v4(p + kOffDO + bx * kBox + r * 128 + ci * 16, make_uint4(0u, 0u, 0u, 0u));
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        __syncthreads();
        if (*sAbort) break;
      }

      // 1. dVN^T = dO^T Aqk + dh^T Kd^T;  meanwhile dh is checkpointed
      if (tid == 0) {
        if (!tc::mbar_wait(&full[slot], par_full)) {
          *sAbort = 1;
        } else {
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tc::umma_bf16(tmem + kColVN, desc_mn(p16 + ((kOffDO + j * 2048) >> 4), kBox),
                          desc_mn(p16 + ((kOffAqk + j * 2048) >> 4), kBox), kIdOA, j > 0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::umma_bf16(tmem + kColVN, desc_mn(sH16 + ((j * 2048) >> 4), kHalfH),
                          desc_k(p16 + ((kOffKd + (j >> 2) * kBox + (j & 3) * 32) >> 4)), kIdHW, 1);
          tc::umma_commit(mma1);
          ++mma1_commits;
        }
      }
      copy_ckpt(c);
      // 2. -dVN^T -> bf16 operand tile
      {
        const bool ok = tc::warp_wait(mma1, par_mma);
        if (ok) {
          tc::tc_fence_after();
          uint32_t x[32];
          tc::tmem_ld32(tlane + kColVN + 32 * half, x);
          tc::tmem_wait_ld();
          unsigned char* vrow = sVN + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 y;
            y.x = pack2<T>(-__uint_as_float(x[8 * q + 0]), -__uint_as_float(x[8 * q + 1]));
            y.y = pack2<T>(-__uint_as_float(x[8 * q + 2]), -__uint_as_float(x[8 * q + 3]));
            y.z = pack2<T>(-__uint_as_float(x[8 * q + 4]), -__uint_as_float(x[8 * q + 5]));
            y.w = pack2<T>(-__uint_as_float(x[8 * q + 6]), -__uint_as_float(x[8 * q + 7]));
            st_shared_v4(vrow + (((4 * half + q) ^ (row & 7)) << 4), y);
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      // 3. dh += Qg^T dO + W^T (-dVN);  meanwhile dVN^T leaves
      if (tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kColH, desc_mn(p16 + ((kOffQg + j * 2048) >> 4), kBox),
                        desc_mn(p16 + ((kOffDO + j * 2048) >> 4), kBox), kIdQO, 1);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kColH, desc_mn(p16 + ((kOffW + j * 2048) >> 4), kBox), desc_k(sVN16 + ((j * 32) >> 4)),
                        kIdKV, 1);
        tc::umma_commit(mma2);
        ++mma2_commits;
      }
      copy_dvn(c);
      // 4. new dh -> bf16 operand tile (the next checkpoint), scaled in place
      //    by the next chunk's 2^G_last; or dh0
      {
        const bool has_next = c - 1 >= c_begin;
        bool ok = tc::warp_wait(mma2, par_mma);
        if (ok && has_next) ok = tc::warp_wait(&full[slot ^ 1], ((i + 1) >> 1) & 1);
        if (ok) {
          tc::tc_fence_after();
          float s[64];
          {
            uint32_t lo[32], hi[32];
            tc::tmem_ld32(tlane + kColH + 64 * half, lo);
            tc::tmem_ld32(tlane + kColH + 64 * half + 32, hi);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) {
              s[e] = __uint_as_float(lo[e]);
              s[32 + e] = __uint_as_float(hi[e]);
            }
          }
          if (has_next) {
            emit_state(s);
            scale_store(s, slot ^ 1);
          } else if (dh0) {
            float4* dst = reinterpret_cast<float4*>(dh0 + (size_t)row * V + 64 * half);
#pragma unroll
            for (int e = 0; e < 16; ++e)
              dst[e] = make_float4(s[4 * e], s[4 * e + 1], s[4 * e + 2], s[4 * e + 3]);
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      if (tid == 0 && c - 2 >= c_begin) issue(c - 2);
    }
  }

  // ---- teardown ---------------------------------------------------------------
  const bool aborted = *sAbort != 0;
  if (aborted && tid == 0) {
    for (int j = c; j > next_issue; --j) {
      const int ij = c_end - 1 - j;
      tc::mbar_wait(&full[ij & 1], (ij >> 1) & 1);
    }
    if (mma1_commits > 0) tc::mbar_wait(mma1, (mma1_commits - 1) & 1);
    if (mma2_commits > 0) tc::mbar_wait(mma2, (mma2_commits - 1) & 1);
    atomicOr(&g_gdn2_fault, 1u);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Forward state pass split over value columns: two CTAs per (sequence, head),
// each owning 64 of the 128 value columns, for launches whose full-width
// grid would leave most SMs idle (B*H well below the SM count).  Each chunk's
// serial chain then carries half the tensor-memory traffic and half the
// products.  Every product keeps M = 128 by stacking:
//   D[0:64)   = W h_half      -> VN = U - W h      (lanes = tokens)
//   D[64:128) = Qg h_half     -> o = Qg h + Aqk VN (lanes = tokens)
//   A = [W ; Qg] (K-major, two 64-row TMA boxes back to back per key half);
//   o: D += [0 ; Aqk] VN      (a zero box in front of Aqk; the upper lanes
//                              only gain zeros)
//   h_half += Kd^T VN         (A = Kd, MN-major; B = VN [t][v], MN-major)
// TMEM: cols [0,64) D, cols [64,128) h_half (lane = key row).  Same rounding
// points as k_fwd_state_tc; VN leaves value-major ([V][64]) as the backward
// reads it.
// ---------------------------------------------------------------------------
constexpr uint32_t kHOffWQ = 0;                 // [W_k0 | Qg_k0 | W_k1 | Qg_k1]
constexpr uint32_t kHOffKd = 4 * kBox;          // [Kd_k0 | Kd_k1]
constexpr uint32_t kHOffZ = 6 * kBox;           // zeros, then Aqk right after
constexpr uint32_t kHOffAqk = 7 * kBox;
constexpr uint32_t kHOffU = 8 * kBox;           // U columns of this half, swizzled
constexpr uint32_t kHOffGl = 9 * kBox;          // [128] fp32
constexpr uint32_t kHSlotBytes = 9 * kBox + 1024;
constexpr uint32_t kHTxBytes = 8 * kBox + kGlBytes;  // the zero box is not copied
constexpr uint32_t kHOffH = 2 * kHSlotBytes;    // bf16 h_half [k][64 v], MN-major (16 KB)
constexpr uint32_t kHOffVN = kHOffH + 2 * kBox; // bf16 VN [t][64 v], MN-major (8 KB)
constexpr uint32_t kHOffVT = kHOffVN + kBox;    // bf16 VN^T [64 v][t], plain (8 KB)
constexpr uint32_t kHOffO = kHOffVT + kBox;     // bf16 o [t][64 v], chunk-swizzled (8 KB)
constexpr uint32_t kHOffBar = kHOffO + kBox;
constexpr uint32_t kHSmemBytes = kHOffBar + 64 + 1024;
constexpr uint32_t kHColD = 0, kHColH = 64, kHTmemCols = 128;
constexpr uint32_t kIdWQh = tc::idesc_bf16(128, 64, 0, 1);  // [W;Qg] h_half, [0;Aqk] VN
constexpr uint32_t kIdKVh = tc::idesc_bf16(128, 64, 1, 1);  // Kd^T VN

__global__ void __launch_bounds__(kTcThreads, 1)
    k_fwd_state_tc_half(FwdStateArgs a, const __grid_constant__ CUtensorMap mW,
                        const __grid_constant__ CUtensorMap mQg,
                        const __grid_constant__ CUtensorMap mKd,
                        const __grid_constant__ CUtensorMap mAqk,
                        const __grid_constant__ CUtensorMap mU) {
  using T = __nv_bfloat16;
  constexpr int K = 128, V = 128;
  extern __shared__ unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kHOffBar);  // [2]
  uint64_t* mma1 = full + 2;
  uint64_t* mma2 = full + 3;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
  unsigned char* sH = sm + kHOffH;
  const uint32_t sH16 = (smem_u32(sm) >> 4) + (kHOffH >> 4);
  unsigned char* sVN = sm + kHOffVN;
  const uint32_t sVN16 = (smem_u32(sm) >> 4) + (kHOffVN >> 4);
  unsigned char* sVT = sm + kHOffVT;
  unsigned char* sO = sm + kHOffO;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;      // the TMEM lane this thread reads
  const int H = a.H;
  const int nh = blockIdx.x >> 1, vh = blockIdx.x & 1, n = nh / H, h = nh - n * H;
  const int v0 = 64 * vh;                // this CTA's value columns [v0, v0 + 64)
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];
  const int64_t bos = a.seqs.cu[n], eos = a.seqs.cu[n + 1];
  const int64_t ldo = (int64_t)H * V;
  const float* h0 = a.h0 ? a.h0 + (int64_t)nh * K * V : nullptr;
  float* ht = a.ht ? a.ht + (int64_t)nh * K * V : nullptr;
  const uint64_t lim = a.wait_ns ? a.wait_ns : tc::kWaitLimitNs;

  if (c_begin >= c_end) {  // empty sequence: the state passes through
    if (ht)
      for (int i = tid; i < K * 64; i += kTcThreads) {
        const int k = i >> 6, v = v0 + (i & 63);
        ht[(size_t)k * V + v] = h0 ? h0[(size_t)k * V + v] : 0.f;
      }
    return;
  }

  // the zero boxes stacked over Aqk (never written by TMA)
  for (int i = tid; i < 2 * (int)(kBox / 16); i += kTcThreads) {
    const int slot = i / (int)(kBox / 16), e = i - slot * (int)(kBox / 16);
    st_shared_v4(sm + slot * kHSlotBytes + kHOffZ + 16 * e, make_uint4(0u, 0u, 0u, 0u));
  }
  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(mma1, 1);
    tc::mbar_init(mma2, 1);
    *sAbort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(sTmem, kHTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *sTmem;
  const uint32_t tlane = tmem + ((uint32_t)(quad * 32) << 16);

  int next_issue = c_begin;
  int mma1_commits = 0, mma2_commits = 0;
  auto issue = [&](int c) {
    if (c == a.skip_chunk) {  // test of the abort path: this chunk never arrives
      next_issue = c + 1;
      return;
    }
    const int slot = (c - c_begin) & 1;
    unsigned char* p = sm + slot * kHSlotBytes;
    const size_t ch = (size_t)c * H + h;
    const int y = (int)(ch * kChunk);
    tc::mbar_expect_tx(&full[slot], kHTxBytes);
    tc::tma_load_2d(p + kHOffWQ, &mW, 0, y, &full[slot]);
    tc::tma_load_2d(p + kHOffWQ + kBox, &mQg, 0, y, &full[slot]);
    tc::tma_load_2d(p + kHOffWQ + 2 * kBox, &mW, 64, y, &full[slot]);
    tc::tma_load_2d(p + kHOffWQ + 3 * kBox, &mQg, 64, y, &full[slot]);
    tc::tma_load_2d(p + kHOffKd, &mKd, 0, y, &full[slot]);
    tc::tma_load_2d(p + kHOffKd + kBox, &mKd, 64, y, &full[slot]);
    tc::tma_load_2d(p + kHOffAqk, &mAqk, 0, y, &full[slot]);
    tc::tma_load_2d(p + kHOffU, &mU, v0, y, &full[slot]);
    tc::bulk_load(p + kHOffGl, a.saved + a.L.gl + ch * K * sizeof(float), kGlBytes, &full[slot]);
    next_issue = c + 1;
  };
  if (tid == 0) {
    issue(c_begin);
    if (c_begin + 1 < c_end) issue(c_begin + 1);
  }

  // bf16 copy of this thread's 32 state values (key row `row`, value columns
  // 32*half ..) into the MN-major operand tile
  auto emit_state = [&](const float (&s)[32]) {
    unsigned char* srow = sH + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 x;
      x.x = pack2<T>(s[8 * q + 0], s[8 * q + 1]);
      x.y = pack2<T>(s[8 * q + 2], s[8 * q + 3]);
      x.z = pack2<T>(s[8 * q + 4], s[8 * q + 5]);
      x.w = pack2<T>(s[8 * q + 6], s[8 * q + 7]);
      st_shared_v4(srow + (((4 * half + q) ^ (row & 7)) << 4), x);
    }
  };
  auto scale_store = [&](const float (&s)[32], int slot) {
    const float gl = reinterpret_cast<const float*>(sm + slot * kHSlotBytes + kHOffGl)[row];
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = s[i] * gl;
    tc::tmem_st32(tlane + kHColH + 32 * half, x);
  };
  auto copy_ckpt = [&](int c) {  // sH -> checkpoint rows, columns [v0, v0 + 64)
    T* gh = reinterpret_cast<T*>(a.saved + a.L.h) + ((size_t)c * H + h) * (size_t)K * V + v0;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = tid + it * kTcThreads;
      const int k = idx >> 3, ci = idx & 7;
      const uint4 x = ld_shared_v4(sH + (k >> 3) * 1024 + (k & 7) * 128 + ((ci ^ (k & 7)) << 4));
      *reinterpret_cast<uint4*>(gh + (size_t)k * V + 8 * ci) = x;
    }
  };
  auto copy_vt = [&](int c) {  // sVT -> VN^T rows [v0, v0 + 64) of chunk c
    T* gv = reinterpret_cast<T*>(a.saved + a.L.vn) + ((size_t)c * H + h) * (size_t)kChunk * V +
            (size_t)v0 * kChunk;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int idx = tid + it * kTcThreads;
      const int v = idx >> 3, ci = idx & 7;
      *reinterpret_cast<uint4*>(gv + (size_t)v * kChunk + 8 * ci) =
          ld_shared_v4(sVT + v * 128 + ci * 16);
    }
  };
  auto copy_o = [&](int c) {  // sO -> output rows of chunk c, columns [v0, v0 + 64)
    const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);
    T* go = reinterpret_cast<T*>(a.o) + cp.row0 * ldo + (int64_t)h * V + v0;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int idx = tid + it * kTcThreads;
      const int t = idx >> 3, ci = idx & 7;
      if (t < cp.len)
        *reinterpret_cast<uint4*>(go + (int64_t)t * ldo + 8 * ci) =
            ld_shared_v4(sO + t * 128 + ((ci ^ (t & 7)) << 4));
    }
  };

  // ---- initial state ----------------------------------------------------------
  {
    const bool ok = tc::warp_wait(&full[0], 0, lim);
    if (ok) {
      float s[32];
      if (h0) {
        const float4* src = reinterpret_cast<const float4*>(h0 + (size_t)row * V + v0 + 32 * half);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 x = src[i];
          s[4 * i] = x.x;
          s[4 * i + 1] = x.y;
          s[4 * i + 2] = x.z;
          s[4 * i + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = 0.f;
      }
      emit_state(s);
      scale_store(s, 0);
    } else if (lane == 0) {
      *sAbort = 1;
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
  }

  int c = c_begin;
  if (!*sAbort) {
    for (; c < c_end; ++c) {
      const int i = c - c_begin, slot = i & 1;
      unsigned char* p = sm + slot * kHSlotBytes;
      const uint32_t p16 = (smem_u32(sm) >> 4) + slot * (kHSlotBytes >> 4);
      const uint32_t par_full = (i >> 1) & 1, par_mma = i & 1;

      // 1. D = [W ; Qg] h_half;  meanwhile the checkpoint of chunk c and the
      //    previous chunk's o leave through the copy units
      if (tid == 0) {
        if (!tc::mbar_wait(&full[slot], par_full, lim)) {
          *sAbort = 1;
        } else {
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::umma_bf16(tmem + kHColD, desc_k(p16 + ((kHOffWQ + (j >> 2) * 2 * kBox + (j & 3) * 32) >> 4)),
                          desc_mn(sH16 + ((j * 2048) >> 4), kBox), kIdWQh, j > 0);
          tc::umma_commit(mma1);
          ++mma1_commits;
        }
      }
      copy_ckpt(c);
      if (c > c_begin) copy_o(c - 1);
      // 2. VN = U - W h (lanes 0-63): bf16 VN [t][v] operand tile and its
      //    value-major copy for the saved buffer
      {
        bool ok = tc::warp_wait(mma1, par_mma, lim);
        if (ok) ok = tc::warp_wait(&full[slot], par_full, lim);
        if (ok && quad < 2) {
          tc::tc_fence_after();
          uint32_t x[32];
          tc::tmem_ld32(tlane + kHColD + 32 * half, x);
          const int t = row;  // token
          uint4 u4[4];
#pragma unroll
          for (int q = 0; q < 4; ++q)
            u4[q] = ld_shared_v4(p + kHOffU + (t >> 3) * 1024 + (t & 7) * 128 +
                                 (((4 * half + q) ^ (t & 7)) << 4));
          tc::tmem_wait_ld();
          unsigned char* vrow = sVN + (t >> 3) * 1024 + (t & 7) * 128;
          T* vt = reinterpret_cast<T*>(sVT) + t;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t uw[4] = {u4[q].x, u4[q].y, u4[q].z, u4[q].w};
            float vn[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 u2 = unpack2<T>(uw[e]);
              vn[2 * e] = u2.x - __uint_as_float(x[8 * q + 2 * e]);
              vn[2 * e + 1] = u2.y - __uint_as_float(x[8 * q + 2 * e + 1]);
            }
            uint4 y;
            y.x = pack2<T>(vn[0], vn[1]);
            y.y = pack2<T>(vn[2], vn[3]);
            y.z = pack2<T>(vn[4], vn[5]);
            y.w = pack2<T>(vn[6], vn[7]);
            st_shared_v4(vrow + (((4 * half + q) ^ (t & 7)) << 4), y);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              vt[(32 * half + 8 * q + e) * kChunk] = from_f<T>(vn[e]);
          }
        }
        if (!ok && lane == 0) *sAbort = 1;
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      // 3. o += [0 ; Aqk] VN,  h_half += Kd^T VN;  meanwhile VN^T leaves
      if (tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kHColD, desc_k(p16 + ((kHOffZ + j * 32) >> 4)), desc_mn(sVN16 + ((j * 2048) >> 4), kBox),
                        kIdWQh, 1);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kHColH, desc_mn(p16 + ((kHOffKd + j * 2048) >> 4), kBox),
                        desc_mn(sVN16 + ((j * 2048) >> 4), kBox), kIdKVh, 1);
        tc::umma_commit(mma2);
        ++mma2_commits;
      }
      copy_vt(c);
      // 4. o (lanes 64-127) -> staging; new state -> bf16 operand tile (the
      //    next checkpoint), scaled in place by the next chunk's 2^G_last
      {
        const bool has_next = c + 1 < c_end;
        bool ok = tc::warp_wait(mma2, par_mma, lim);
        if (ok && has_next) ok = tc::warp_wait(&full[slot ^ 1], ((i + 1) >> 1) & 1, lim);
        if (ok) {
          tc::tc_fence_after();
          if (quad >= 2) {
            uint32_t x[32];
            tc::tmem_ld32(tlane + kHColD + 32 * half, x);
            tc::tmem_wait_ld();
            const int t = row - 64;
            unsigned char* orow = sO + t * 128;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              uint4 y;
              y.x = pack2<T>(__uint_as_float(x[8 * q + 0]), __uint_as_float(x[8 * q + 1]));
              y.y = pack2<T>(__uint_as_float(x[8 * q + 2]), __uint_as_float(x[8 * q + 3]));
              y.z = pack2<T>(__uint_as_float(x[8 * q + 4]), __uint_as_float(x[8 * q + 5]));
              y.w = pack2<T>(__uint_as_float(x[8 * q + 6]), __uint_as_float(x[8 * q + 7]));
              st_shared_v4(orow + (((4 * half + q) ^ (t & 7)) << 4), y);
            }
          }
          float s[32];
          {
            uint32_t hx[32];
            tc::tmem_ld32(tlane + kHColH + 32 * half, hx);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) s[e] = __uint_as_float(hx[e]);
          }
          if (has_next) {
            emit_state(s);
            scale_store(s, slot ^ 1);
          } else if (ht) {
            float4* dst = reinterpret_cast<float4*>(ht + (size_t)row * V + v0 + 32 * half);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              dst[e] = make_float4(s[4 * e], s[4 * e + 1], s[4 * e + 2], s[4 * e + 3]);
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      if (tid == 0 && c + 2 < c_end) issue(c + 2);
    }
  }

  // ---- teardown ---------------------------------------------------------------
  const bool aborted = *sAbort != 0;
  if (!aborted) copy_o(c_end - 1);
  if (aborted && tid == 0) {
    for (int j = c; j < next_issue; ++j) {
      const int ij = j - c_begin;
      tc::mbar_wait(&full[ij & 1], (ij >> 1) & 1, lim);
    }
    if (mma1_commits > 0) tc::mbar_wait(mma1, (mma1_commits - 1) & 1, lim);
    if (mma2_commits > 0) tc::mbar_wait(mma2, (mma2_commits - 1) & 1, lim);
    atomicOr(&g_gdn2_fault, 1u);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kHTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Backward state pass split over value columns (as k_fwd_state_tc_half):
// two CTAs per (sequence, head), 64 value columns each.  Products keep
// M = 128 by stacking zero boxes under the token-major operands:
//   D[0:64) = dVN_half = Aqk^T dO_half + Kd dh_half   (lanes = tokens)
//     A = [Aqk^T ; 0] (MN-major, the zero box one M-atom further) and
//     A = [Kd ; 0]    (K-major, a zero box after each Kd key-half box)
//   dh_half += Qg^T dO_half + W^T (-dVN_half)          (lanes = key rows)
// TMEM: cols [0,64) D, cols [64,128) dh_half.  Same rounding points as
// k_bwd_state_tc; dVN leaves value-major ([V][64]).
// ---------------------------------------------------------------------------
constexpr uint32_t kBOffAZ = 0;                  // [Aqk | 0]
constexpr uint32_t kBOffKZ = 2 * kBox;           // [Kd_k0 | 0 | Kd_k1 | 0]
constexpr uint32_t kBOffQg = 6 * kBox;           // [Qg_k0 | Qg_k1]
constexpr uint32_t kBOffW = 8 * kBox;            // [W_k0 | W_k1]
constexpr uint32_t kBOffDO = 10 * kBox;          // dO columns of this half, swizzled
constexpr uint32_t kBOffGl = 11 * kBox;          // [128] fp32
constexpr uint32_t kBSlotBytes = 11 * kBox + 1024;
constexpr uint32_t kBTxBytes = 8 * kBox + kGlBytes;  // zero boxes are not copied
constexpr uint32_t kBOffH = 2 * kBSlotBytes;     // bf16 dh_half [k][64 v], MN-major (16 KB)
constexpr uint32_t kBOffVN = kBOffH + 2 * kBox;  // bf16 -dVN [t][64 v], MN-major (8 KB)
constexpr uint32_t kBOffVT = kBOffVN + kBox;     // bf16 dVN^T [64 v][t], plain (8 KB)
constexpr uint32_t kBOffBar = kBOffVT + kBox;
constexpr uint32_t kBSmemBytes = kBOffBar + 64 + 1024;
constexpr uint32_t kIdMNh = tc::idesc_bf16(128, 64, 1, 1);  // MN-major A, MN-major B
constexpr uint32_t kIdKNh = tc::idesc_bf16(128, 64, 0, 1);  // K-major A, MN-major B

__global__ void __launch_bounds__(kTcThreads, 1)
    k_bwd_state_tc_half(BwdStateArgs a, const __grid_constant__ CUtensorMap mW,
                        const __grid_constant__ CUtensorMap mQg,
                        const __grid_constant__ CUtensorMap mKd,
                        const __grid_constant__ CUtensorMap mAqk,
                        const __grid_constant__ CUtensorMap mDO) {
  using T = __nv_bfloat16;
  constexpr int K = 128, V = 128;
  extern __shared__ unsigned char smraw[];
  unsigned char* sm = smraw + ((1024u - (smem_u32(smraw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kBOffBar);  // [2]
  uint64_t* mma1 = full + 2;
  uint64_t* mma2 = full + 3;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(full + 4);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sTmem + 1);
  unsigned char* sH = sm + kBOffH;
  const uint32_t sH16 = (smem_u32(sm) >> 4) + (kBOffH >> 4);
  unsigned char* sVN = sm + kBOffVN;
  const uint32_t sVN16 = (smem_u32(sm) >> 4) + (kBOffVN >> 4);
  unsigned char* sVT = sm + kBOffVT;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quad = warp & 3, half = warp >> 2;
  const int row = quad * 32 + lane;
  const int H = a.H;
  const int nh = blockIdx.x >> 1, vh = blockIdx.x & 1, n = nh / H, h = nh - n * H;
  const int v0 = 64 * vh;
  const int c_begin = a.seqs.coff[n], c_end = a.seqs.coff[n + 1];
  const int64_t bos = a.seqs.cu[n], eos = a.seqs.cu[n + 1];
  const float* dht = a.dht ? a.dht + (int64_t)nh * K * V : nullptr;
  float* dh0 = a.dh0 ? a.dh0 + (int64_t)nh * K * V : nullptr;

  if (c_begin >= c_end) {  // empty sequence: the gradient passes through
    if (dh0)
      for (int i = tid; i < K * 64; i += kTcThreads) {
        const int k = i >> 6, v = v0 + (i & 63);
        dh0[(size_t)k * V + v] = dht ? dht[(size_t)k * V + v] : 0.f;
      }
    return;
  }

  // zero boxes stacked under Aqk^T and Kd (never written by TMA)
  for (int i = tid; i < 2 * 3 * (int)(kBox / 16); i += kTcThreads) {
    const int slot = i / (3 * (int)(kBox / 16)), e = i - slot * 3 * (int)(kBox / 16);
    const int box = e / (int)(kBox / 16), o = e - box * (int)(kBox / 16);
    const uint32_t off = box == 0 ? kBOffAZ + kBox : (box == 1 ? kBOffKZ + kBox : kBOffKZ + 3 * kBox);
    st_shared_v4(sm + slot * kBSlotBytes + off + 16 * o, make_uint4(0u, 0u, 0u, 0u));
  }
  if (tid == 0) {
    tc::mbar_init(&full[0], 1);
    tc::mbar_init(&full[1], 1);
    tc::mbar_init(mma1, 1);
    tc::mbar_init(mma2, 1);
    *sAbort = 0;
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(sTmem, kHTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_async_smem();
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *sTmem;
  const uint32_t tlane = tmem + ((uint32_t)(quad * 32) << 16);

  // chunk c sits in slot (c_end - 1 - c) & 1
  int next_issue = c_end - 1;
  int mma1_commits = 0, mma2_commits = 0;
  auto issue = [&](int c) {
    const int slot = (c_end - 1 - c) & 1;
    unsigned char* p = sm + slot * kBSlotBytes;
    const size_t ch = (size_t)c * H + h;
    const int y = (int)(ch * kChunk);
    const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);
    tc::mbar_expect_tx(&full[slot], kBTxBytes);
    tc::tma_load_2d(p + kBOffAZ, &mAqk, 0, y, &full[slot]);
    tc::tma_load_2d(p + kBOffKZ, &mKd, 0, y, &full[slot]);
    tc::tma_load_2d(p + kBOffKZ + 2 * kBox, &mKd, 64, y, &full[slot]);
    tc::tma_load_2d(p + kBOffQg, &mQg, 0, y, &full[slot]);
    tc::tma_load_2d(p + kBOffQg + kBox, &mQg, 64, y, &full[slot]);
    tc::tma_load_2d(p + kBOffW, &mW, 0, y, &full[slot]);
    tc::tma_load_2d(p + kBOffW + kBox, &mW, 64, y, &full[slot]);
    tc::tma_load_3d(p + kBOffDO, &mDO, v0, h, (int)cp.row0, &full[slot]);
    tc::bulk_load(p + kBOffGl, a.saved + a.L.gl + ch * K * sizeof(float), kGlBytes, &full[slot]);
    next_issue = c - 1;
  };
  if (tid == 0) {
    issue(c_end - 1);
    if (c_end - 2 >= c_begin) issue(c_end - 2);
  }

  auto emit_state = [&](const float (&s)[32]) {
    unsigned char* srow = sH + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 x;
      x.x = pack2<T>(s[8 * q + 0], s[8 * q + 1]);
      x.y = pack2<T>(s[8 * q + 2], s[8 * q + 3]);
      x.z = pack2<T>(s[8 * q + 4], s[8 * q + 5]);
      x.w = pack2<T>(s[8 * q + 6], s[8 * q + 7]);
      st_shared_v4(srow + (((4 * half + q) ^ (row & 7)) << 4), x);
    }
  };
  auto scale_store = [&](const float (&s)[32], int slot) {
    const float gl = reinterpret_cast<const float*>(sm + slot * kBSlotBytes + kBOffGl)[row];
    float x[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = s[i] * gl;
    tc::tmem_st32(tlane + kHColH + 32 * half, x);
  };
  auto copy_ckpt = [&](int c) {  // sH -> dh of chunk c, columns [v0, v0 + 64)
    T* gh = reinterpret_cast<T*>(a.ws + a.BL.dh) + ((size_t)c * H + h) * (size_t)K * V + v0;
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int idx = tid + it * kTcThreads;
      const int k = idx >> 3, ci = idx & 7;
      const uint4 x = ld_shared_v4(sH + (k >> 3) * 1024 + (k & 7) * 128 + ((ci ^ (k & 7)) << 4));
      *reinterpret_cast<uint4*>(gh + (size_t)k * V + 8 * ci) = x;
    }
  };
  auto copy_dvt = [&](int c) {  // sVT -> dVN^T rows [v0, v0 + 64) of chunk c
    T* gv = reinterpret_cast<T*>(a.ws + a.BL.dvn) + ((size_t)c * H + h) * (size_t)kChunk * V +
            (size_t)v0 * kChunk;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
      const int idx = tid + it * kTcThreads;
      const int v = idx >> 3, ci = idx & 7;
      *reinterpret_cast<uint4*>(gv + (size_t)v * kChunk + 8 * ci) =
          ld_shared_v4(sVT + v * 128 + ci * 16);
    }
  };

  // ---- initial gradient -----------------------------------------------------
  {
    const bool ok = tc::warp_wait(&full[0], 0);
    if (ok) {
      float s[32];
      if (dht) {
        const float4* src = reinterpret_cast<const float4*>(dht + (size_t)row * V + v0 + 32 * half);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 x = src[i];
          s[4 * i] = x.x;
          s[4 * i + 1] = x.y;
          s[4 * i + 2] = x.z;
          s[4 * i + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) s[i] = 0.f;
      }
      emit_state(s);
      scale_store(s, 0);
    } else if (lane == 0) {
      *sAbort = 1;
    }
    tc::fence_async_smem();
    tc::tc_fence_before();
    __syncthreads();
  }

  int c = c_end - 1;
  if (!*sAbort) {
    for (; c >= c_begin; --c) {
      const int i = c_end - 1 - c, slot = i & 1;
      unsigned char* p = sm + slot * kBSlotBytes;
      const uint32_t p16 = (smem_u32(sm) >> 4) + slot * (kBSlotBytes >> 4);
      const uint32_t par_full = (i >> 1) & 1, par_mma = i & 1;
      const ChunkPos cp = chunk_pos_in_seq(bos, eos, c_begin, c);

      // 0. a partial chunk's dO rows past the sequence end belong to the
      //    next sequence: zero them before any product reads the tile
      if (cp.len < kChunk) {
        const bool ok = tc::warp_wait(&full[slot], par_full);
        if (ok) {
          for (int e = tid; e < (kChunk - cp.len) * 8; e += kTcThreads) {
            const int r = cp.len + (e >> 3), ci = e & 7;
            st_shared_v4(p + kBOffDO + r * 128 + ci * 16, make_uint4(0u, 0u, 0u, 0u));
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        __syncthreads();
        if (*sAbort) break;
      }

      // 1. dVN_half = Aqk^T dO_half + Kd dh_half;  meanwhile dh is checkpointed
      if (tid == 0) {
        if (!tc::mbar_wait(&full[slot], par_full)) {
          *sAbort = 1;
        } else {
          tc::tc_fence_after();
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tc::umma_bf16(tmem + kHColD, desc_mn(p16 + ((kBOffAZ + j * 2048) >> 4), kBox),
                          desc_mn(p16 + ((kBOffDO + j * 2048) >> 4), kBox), kIdMNh, j > 0);
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::umma_bf16(tmem + kHColD, desc_k(p16 + ((kBOffKZ + (j >> 2) * 2 * kBox + (j & 3) * 32) >> 4)),
                          desc_mn(sH16 + ((j * 2048) >> 4), kBox), kIdKNh, 1);
          tc::umma_commit(mma1);
          ++mma1_commits;
        }
      }
      copy_ckpt(c);
      // 2. -dVN [t][v] -> bf16 operand tile; dVN^T -> staging (lanes 0-63)
      {
        const bool ok = tc::warp_wait(mma1, par_mma);
        if (ok && quad < 2) {
          tc::tc_fence_after();
          uint32_t x[32];
          tc::tmem_ld32(tlane + kHColD + 32 * half, x);
          tc::tmem_wait_ld();
          const int t = row;
          unsigned char* vrow = sVN + (t >> 3) * 1024 + (t & 7) * 128;
          T* vt = reinterpret_cast<T*>(sVT) + t;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 y;
            y.x = pack2<T>(-__uint_as_float(x[8 * q + 0]), -__uint_as_float(x[8 * q + 1]));
            y.y = pack2<T>(-__uint_as_float(x[8 * q + 2]), -__uint_as_float(x[8 * q + 3]));
            y.z = pack2<T>(-__uint_as_float(x[8 * q + 4]), -__uint_as_float(x[8 * q + 5]));
            y.w = pack2<T>(-__uint_as_float(x[8 * q + 6]), -__uint_as_float(x[8 * q + 7]));
            st_shared_v4(vrow + (((4 * half + q) ^ (t & 7)) << 4), y);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              vt[(32 * half + 8 * q + e) * kChunk] = from_f<T>(__uint_as_float(x[8 * q + e]));
          }
        }
        if (!ok && lane == 0) *sAbort = 1;
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      // 3. dh_half += Qg^T dO_half + W^T (-dVN_half);  meanwhile dVN^T leaves
      if (tid == 0) {
        tc::tc_fence_after();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kHColH, desc_mn(p16 + ((kBOffQg + j * 2048) >> 4), kBox),
                        desc_mn(p16 + ((kBOffDO + j * 2048) >> 4), kBox), kIdMNh, 1);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::umma_bf16(tmem + kHColH, desc_mn(p16 + ((kBOffW + j * 2048) >> 4), kBox),
                        desc_mn(sVN16 + ((j * 2048) >> 4), kBox), kIdMNh, 1);
        tc::umma_commit(mma2);
        ++mma2_commits;
      }
      copy_dvt(c);
      // 4. new dh_half -> bf16 operand tile (the next checkpoint), scaled in
      //    place by the next chunk's 2^G_last; or dh0
      {
        const bool has_next = c - 1 >= c_begin;
        bool ok = tc::warp_wait(mma2, par_mma);
        if (ok && has_next) ok = tc::warp_wait(&full[slot ^ 1], ((i + 1) >> 1) & 1);
        if (ok) {
          tc::tc_fence_after();
          float s[32];
          {
            uint32_t hx[32];
            tc::tmem_ld32(tlane + kHColH + 32 * half, hx);
            tc::tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) s[e] = __uint_as_float(hx[e]);
          }
          if (has_next) {
            emit_state(s);
            scale_store(s, slot ^ 1);
          } else if (dh0) {
            float4* dst = reinterpret_cast<float4*>(dh0 + (size_t)row * V + v0 + 32 * half);
#pragma unroll
            for (int e = 0; e < 8; ++e)
              dst[e] = make_float4(s[4 * e], s[4 * e + 1], s[4 * e + 2], s[4 * e + 3]);
          }
        } else if (lane == 0) {
          *sAbort = 1;
        }
        tc::fence_async_smem();
        tc::tc_fence_before();
        __syncthreads();
        if (*sAbort) break;
      }
      if (tid == 0 && c - 2 >= c_begin) issue(c - 2);
    }
  }

  // ---- teardown ---------------------------------------------------------------
  const bool aborted = *sAbort != 0;
  if (aborted && tid == 0) {
    for (int j = c; j > next_issue; --j) {
      const int ij = c_end - 1 - j;
      tc::mbar_wait(&full[ij & 1], (ij >> 1) & 1);
    }
    if (mma1_commits > 0) tc::mbar_wait(mma1, (mma1_commits - 1) & 1);
    if (mma2_commits > 0) tc::mbar_wait(mma2, (mma2_commits - 1) & 1);
    atomicOr(&g_gdn2_fault, 1u);
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, kHTmemCols);
  }
}

// ---- host side -----------------------------------------------------------------
bool make_map(CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint32_t box_x,
              bool swizzle) {
  return tmap_2d_bf16(m, base, inner, rows, box_x, swizzle);
}
bool make_map_rows(CUtensorMap* m, const void* base, uint64_t V, uint64_t H, uint64_t rows) {
  return tmap_rows(m, base, V, H, rows, 64, 2);
}
bool encode_ok() { return tmap_available(); }

}  // namespace

// True when k_bwd_state_tc can serve the problem (bf16, K = V = 128, no
// pre-scan, 16-byte aligned buffers, TMA-addressable rows).
bool bwd_state_tc_ok(const BwdStateArgs& a, int dtype_bf16) {
  if (!dtype_bf16 || a.K != 128 || a.V != 128 || a.prescan || !a.dout || !a.ws) return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.saved) | reinterpret_cast<uintptr_t>(a.ws) |
                       reinterpret_cast<uintptr_t>(a.dout) | reinterpret_cast<uintptr_t>(a.dht) |
                       reinterpret_cast<uintptr_t>(a.dh0);
  if ((al & 15) != 0) return false;
  if ((int64_t)a.seqs.n_chunks * a.H * kChunk >= (int64_t)1 << 31) return false;
  if (a.total_rows <= 0 || a.total_rows >= (int64_t)1 << 31) return false;
  return encode_ok();
}

cudaError_t launch_bwd_state_tc(const BwdStateArgs& a, cudaStream_t st) {
  const uint64_t rows = (uint64_t)a.seqs.n_chunks * a.H * kChunk;
  CUtensorMap mW, mQg, mKd, mAqk, mDO;
  if (!make_map(&mW, a.saved + a.L.w, 128, rows, 64, true) ||
      !make_map(&mQg, a.saved + a.L.qg, 128, rows, 64, true) ||
      !make_map(&mKd, a.saved + a.L.kd, 128, rows, 64, true) ||
      !make_map(&mAqk, a.saved + a.L.aqk, 64, rows, 64, true) ||
      !make_map_rows(&mDO, a.dout, 128, (uint64_t)a.H, (uint64_t)a.total_rows))
    return cudaErrorInvalidValue;
  const int grid = a.seqs.n_seqs * a.H;
  if (grid == 0) return cudaSuccess;
  int sms = 0;
  cudaError_t e = num_sms(&sms);
  if (e != cudaSuccess) return e;
  if (a.max_ctas > 0 && a.max_ctas < sms) sms = a.max_ctas;
  if (2 * grid <= sms) {  // few sequence-heads: one CTA per half of the value columns
    e = cudaFuncSetAttribute(k_bwd_state_tc_half, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kBSmemBytes);
    if (e != cudaSuccess) return e;
    k_bwd_state_tc_half<<<2 * grid, kTcThreads, kBSmemBytes, st>>>(a, mW, mQg, mKd, mAqk, mDO);
    return cudaGetLastError();
  }
  e = cudaFuncSetAttribute(k_bwd_state_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  k_bwd_state_tc<<<grid, kTcThreads, kSmemBytes, st>>>(a, mW, mQg, mKd, mAqk, mDO);
  return cudaGetLastError();
}

// True when k_fwd_state_tc can serve the problem (bf16, K = V = 128, no
// pre-scan, 16-byte aligned saved buffer, tile rows addressable by TMA).
bool fwd_state_tc_ok(const FwdStateArgs& a, int dtype_bf16) {
  if (!dtype_bf16 || a.K != 128 || a.V != 128 || a.prescan || !a.o) return false;
  if ((reinterpret_cast<uintptr_t>(a.saved) & 15) != 0) return false;
  if ((reinterpret_cast<uintptr_t>(a.h0) & 15) != 0 || (reinterpret_cast<uintptr_t>(a.ht) & 15) != 0)
    return false;
  if ((int64_t)a.seqs.n_chunks * a.H * kChunk >= (int64_t)1 << 31) return false;
  return encode_ok();
}

cudaError_t launch_fwd_state_tc(const FwdStateArgs& a, cudaStream_t st) {
  const uint64_t rows = (uint64_t)a.seqs.n_chunks * a.H * kChunk;
  CUtensorMap mW, mQg, mKd, mAqk, mU;
  if (!make_map(&mW, a.saved + a.L.w, 128, rows, 64, true) ||
      !make_map(&mQg, a.saved + a.L.qg, 128, rows, 64, true) ||
      !make_map(&mKd, a.saved + a.L.kd, 128, rows, 64, true) ||
      !make_map(&mAqk, a.saved + a.L.aqk, 64, rows, 64, true) ||
      !make_map(&mU, a.saved + a.L.u, 128, rows, 128, false))
    return cudaErrorInvalidValue;
  const int grid = a.seqs.n_seqs * a.H;
  if (grid == 0) return cudaSuccess;
  int sms = 0;
  cudaError_t e = num_sms(&sms);
  if (e != cudaSuccess) return e;
  if (a.max_ctas > 0 && a.max_ctas < sms) sms = a.max_ctas;
  if (2 * grid <= sms) {
    // few sequence-heads: two CTAs each, one per half of the value columns
    CUtensorMap mUh;
    if (!make_map(&mUh, a.saved + a.L.u, 128, rows, 64, true)) return cudaErrorInvalidValue;
    e = cudaFuncSetAttribute(k_fwd_state_tc_half, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kHSmemBytes);
    if (e != cudaSuccess) return e;
    k_fwd_state_tc_half<<<2 * grid, kTcThreads, kHSmemBytes, st>>>(a, mW, mQg, mKd, mAqk, mUh);
    return cudaGetLastError();
  }
  e = cudaFuncSetAttribute(k_fwd_state_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)kSmemBytes);
  if (e != cudaSuccess) return e;
  k_fwd_state_tc<<<grid, kTcThreads, kSmemBytes, st>>>(a, mW, mQg, mKd, mAqk, mU);
  return cudaGetLastError();
}

// Address of the fault word on the current device (looked up once per
// device; kernels of other translation units receive it as an argument).
cudaError_t fault_word(unsigned int** ptr) {
  constexpr int kMaxDev = 64;
  static unsigned int* cache[kMaxDev] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDev && cache[dev]) {
    *ptr = cache[dev];
    return cudaSuccess;
  }
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_gdn2_fault);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < kMaxDev) cache[dev] = static_cast<unsigned int*>(p);
  *ptr = static_cast<unsigned int*>(p);
  return cudaSuccess;
}

// Fault bits recorded by bounded waits that ran out (device of the current
// context); `clear` resets them.
cudaError_t read_fault_bits(unsigned int* bits, bool clear) {
  cudaError_t e = cudaMemcpyFromSymbol(bits, g_gdn2_fault, sizeof(unsigned int));
  if (e != cudaSuccess || !clear) return e;
  const unsigned int zero = 0;
  return cudaMemcpyToSymbol(g_gdn2_fault, &zero, sizeof(unsigned int));
}

}  // namespace gdn2
