// common.cuh -- shared device helpers for the GDN-2 B200 kernels.
//
// * element conversion for the three token dtypes (fp32, bf16, fp16);
// * warp-level tensor-core tiles: mma.sync m16n8k8 TF32 with fp32 accumulate,
//   single pass for 16-bit inputs and a 3-term split (hi*hi + hi*lo + lo*hi)
//   for fp32 inputs, reading operands from shared memory through arbitrary
//   (row, column) strides so transposed views cost nothing;
// * chunk geometry (sequence / chunk tables) and the layout of the buffers
//   the forward saves for the backward.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn2 {

constexpr int kChunk = 64;     // chunk length (chunk_gdn2.py:2362 hard-codes 64)
constexpr int kThreads = 256;  // 8 warps per CTA in every chunk kernel
constexpr int kBV = 32;        // value columns per CTA in the state passes
constexpr float kLog2e = 1.4426950408889634f;
// Largest chunk-local log2 decay range inside one 16-row block for which the
// factored (tensor-core) form of the diagonal score blocks stays inside the
// fp32 exponent range; beyond it the exact elementwise form is used.
constexpr float kSafeLog2Range = 100.0f;
constexpr float kNormEps = 1e-6f;  // FLA l2norm eps (fla/modules/l2norm.py)

// ---------------------------------------------------------------------------
// element conversion
// ---------------------------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

// Number of MMA passes: fp32 inputs get the 3-term TF32 split, which keeps
// ~fp32 accuracy; 16-bit inputs carry < 11 mantissa bits so one pass suffices.
template <typename T> struct Passes { static constexpr int value = 1; };
template <> struct Passes<float> { static constexpr int value = 3; };

// ---------------------------------------------------------------------------
// tensor-core tile primitive
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t tf32_bits(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <int MT, int NT>
__device__ __forceinline__ void acc_zero(float (&acc)[MT][NT][4]) {
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
}

// acc[(16*MT) x (8*NT)] += A[(16*MT) x kd] * B[kd x (8*NT)]
//   A(m,k) = A[m*sam + k*sak],  B(k,n) = B[k*sbk + n*sbn]   (shared memory)
// kd must be a multiple of 8.  Every lane of the warp must call this.
template <int MT, int NT, int P>
__device__ __forceinline__ void warp_mma(float (&acc)[MT][NT][4], const float* A, int sam, int sak,
                                         const float* B, int sbk, int sbn, int kd) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  for (int k0 = 0; k0 < kd; k0 += 8) {
    uint32_t ah[MT][4], al[MT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      const float* a = A + (i * 16 + gid) * sam + (k0 + tig) * sak;
      float x[4] = {a[0], a[8 * sam], a[4 * sak], a[8 * sam + 4 * sak]};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ah[i][e] = tf32_bits(x[e]);
        if (P > 1) al[i][e] = tf32_bits(x[e] - __uint_as_float(ah[i][e]));
      }
    }
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float* bp = B + (k0 + tig) * sbk + (j * 8 + gid) * sbn;
      float y0 = bp[0], y1 = bp[4 * sbk];
      uint32_t bh0 = tf32_bits(y0), bh1 = tf32_bits(y1);
      if (P > 1) {
        uint32_t bl0 = tf32_bits(y0 - __uint_as_float(bh0));
        uint32_t bl1 = tf32_bits(y1 - __uint_as_float(bh1));
#pragma unroll
        for (int i = 0; i < MT; ++i) {
          mma_tf32(acc[i][j], al[i], bh0, bh1);
          mma_tf32(acc[i][j], ah[i], bl0, bl1);
        }
      }
#pragma unroll
      for (int i = 0; i < MT; ++i) mma_tf32(acc[i][j], ah[i], bh0, bh1);
    }
  }
}

// Visit every accumulator element with its (row, col) inside the warp tile.
template <int MT, int NT, typename F>
__device__ __forceinline__ void acc_foreach(float (&acc)[MT][NT][4], F&& f) {
  const int lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int i = 0; i < MT; ++i)
#pragma unroll
    for (int j = 0; j < NT; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        f(i * 16 + gid + ((e >> 1) << 3), j * 8 + 2 * tig + (e & 1), acc[i][j][e]);
}

// ---------------------------------------------------------------------------
// tile movement between global token tensors and shared memory
// ---------------------------------------------------------------------------
// Load a ROWS x COLS tile of a [rows, ldg] global view into a float shared
// tile (row stride lds, a multiple of 4).  Rows >= nrows and cols >= ncols
// are zero-filled.  Every thread first issues all of its 16-byte loads
// (ITERS of them, unrolled) and only then converts and stores, so a tile
// costs one memory round trip instead of one per element.  Falls back to
// element loads (still batched) when the view is not 16-byte aligned.
template <typename T, int ROWS, int COLS>
__device__ __forceinline__ void load_tile(float* __restrict__ s, int lds, const T* __restrict__ g,
                                          int64_t ldg, int nrows, int ncols) {
  constexpr int VEC = 16 / sizeof(T);
  static_assert(COLS % VEC == 0, "tile width must be a multiple of 16 bytes");
  constexpr int CPR = COLS / VEC;
  constexpr int TOTAL = ROWS * CPR;
  constexpr int ITERS = (TOTAL + kThreads - 1) / kThreads;
  const bool vec = ((ncols % VEC) == 0) && ((ldg % VEC) == 0) &&
                   ((reinterpret_cast<uintptr_t>(g) & 15) == 0);
  uint4 buf[ITERS];
  if (vec) {
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const int idx = threadIdx.x + it * kThreads;
      const int r = idx / CPR, c = (idx - r * CPR) * VEC;
      buf[it] = make_uint4(0u, 0u, 0u, 0u);
      if (idx < TOTAL && r < nrows && c < ncols)
        buf[it] = __ldg(reinterpret_cast<const uint4*>(g + (int64_t)r * ldg + c));
    }
  } else {
#pragma unroll
    for (int it = 0; it < ITERS; ++it) {
      const int idx = threadIdx.x + it * kThreads;
      const int r = idx / CPR, c = (idx - r * CPR) * VEC;
      T tmp[VEC];
#pragma unroll
      for (int e = 0; e < VEC; ++e) {
        tmp[e] = from_f<T>(0.f);
        if (idx < TOTAL && r < nrows && c + e < ncols) tmp[e] = g[(int64_t)r * ldg + c + e];
      }
      buf[it] = *reinterpret_cast<uint4*>(tmp);
    }
  }
#pragma unroll
  for (int it = 0; it < ITERS; ++it) {
    const int idx = threadIdx.x + it * kThreads;
    if (idx < TOTAL) {
      const int r = idx / CPR, c = (idx - r * CPR) * VEC;
      const T* e = reinterpret_cast<const T*>(&buf[it]);
      float* d = s + r * lds + c;
#pragma unroll
      for (int j = 0; j < VEC; j += 4)
        *reinterpret_cast<float4*>(d + j) =
            make_float4(to_f<T>(e[j]), to_f<T>(e[j + 1]), to_f<T>(e[j + 2]), to_f<T>(e[j + 3]));
    }
  }
}

// In-place inclusive scan down the rows of a 64 x NC float tile (row stride
// lds): prefix sums when REV is false, suffix sums when REV is true.  Same
// segmented scheme as col_cumsum64; `tmp` needs 256 floats.
template <int NC, bool REV>
__device__ __forceinline__ void col_scan64(float* s, int lds, float* tmp) {
  constexpr int NSEG = kThreads / NC;
  constexpr int RPS = kChunk / NSEG;
  const int col = threadIdx.x % NC, seg = threadIdx.x / NC;
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    const int r = REV ? (kChunk - 1 - (seg * RPS + i)) : (seg * RPS + i);
    float* p = s + r * lds + col;
    run += *p;
    *p = run;
  }
  tmp[seg * NC + col] = run;
  __syncthreads();
  float off = 0.f;
  for (int j = 0; j < seg; ++j) off += tmp[j * NC + col];
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    const int r = REV ? (kChunk - 1 - (seg * RPS + i)) : (seg * RPS + i);
    s[r * lds + col] += off;
  }
  __syncthreads();
}

// In-place inclusive prefix sum down the rows of a 64 x NC float tile
// (row stride lds), times `mul`.  The 256 threads split into NC columns x
// (256/NC) row segments: each segment scans its rows, segment totals are
// exchanged through `tmp` (>= 256 floats), then offsets are added.
template <int NC>
__device__ __forceinline__ void col_cumsum64(float* s, int lds, float mul, float* tmp) {
  constexpr int NSEG = kThreads / NC;
  constexpr int RPS = kChunk / NSEG;
  const int col = threadIdx.x % NC, seg = threadIdx.x / NC;
  float run = 0.f;
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    float* p = s + (seg * RPS + i) * lds + col;
    run += *p;
    *p = run;
  }
  tmp[seg * NC + col] = run;
  __syncthreads();
  float off = 0.f;
  for (int j = 0; j < seg; ++j) off += tmp[j * NC + col];
#pragma unroll
  for (int i = 0; i < RPS; ++i) {
    float* p = s + (seg * RPS + i) * lds + col;
    *p = (*p + off) * mul;
  }
  __syncthreads();
}

// 2^x with the hardware base-2 exponential (PTX ex2.approx.ftz.f32: relative
// error about 2^-22; results below 2^-126 flush to zero, far below what the
// 16-bit operands it scales can hold).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Number of SMs of the current device (persistent-kernel grids).
inline cudaError_t num_sms(int* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  return cudaDeviceGetAttribute(out, cudaDevAttrMultiProcessorCount, dev);
}

// ---------------------------------------------------------------------------
// geometry
// ---------------------------------------------------------------------------
struct Seqs {
  const int32_t* cu;      // [N+1] token offsets
  const int32_t* coff;    // [N+1] chunk offsets
  const int32_t* cseq;    // [n_chunks] owning sequence
  int n_seqs, n_chunks;
};

struct ChunkPos {
  int64_t row0;  // first token row of the chunk
  int len;       // valid rows (1..64)
};

// Position of chunk c of a sequence whose first token row is bos, whose end
// row is eos and whose first chunk is c0 (no table lookups).
__device__ __forceinline__ ChunkPos chunk_pos_in_seq(int64_t bos, int64_t eos, int c0, int c) {
  ChunkPos p;
  p.row0 = bos + (int64_t)(c - c0) * kChunk;
  const int64_t rem = eos - p.row0;
  p.len = rem < kChunk ? (int)rem : kChunk;
  return p;
}

__device__ __forceinline__ ChunkPos chunk_pos(const Seqs& s, int c) {
  int n = s.cseq[c];
  int j = c - s.coff[n];
  int64_t bos = s.cu[n];
  int64_t eos = s.cu[n + 1];
  ChunkPos p;
  p.row0 = bos + (int64_t)j * kChunk;
  int64_t rem = eos - p.row0;
  p.len = rem < kChunk ? (int)rem : kChunk;
  return p;
}

// Layout of the buffer the forward fills for the backward.  Per (chunk, head):
//   Qg, Kd, W : [64][K]  (T)   scale*q*2^G,  k*2^(G_last-G),  A (b*k*2^G)
//   U         : [64][V]  (T)   A (w*v)
//   VN        : [64][V]  (T)   U - W h;  stored transposed, [V][64], by the
//                              bf16 tensor-core path (state16.cu,
//                              state_tc.cu -> bwd16.cu)
//   Aqk, A    : [64][64] (T)   causal scores (scale folded in), (I+Akk)^-1
//   gl        : [K]      (f32) 2^G_last
//   h         : [K][V]   (T)   state entering the chunk
// Offsets are in bytes; each section starts on a 256-byte boundary.
struct SavedLayout {
  size_t qg, kd, w, u, vn, aqk, a, gl, h, total;
};

__host__ __device__ inline size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

__host__ __device__ inline SavedLayout saved_layout(int64_t n_chunks, int H, int K, int V,
                                                    int esize) {
  SavedLayout L;
  size_t nh = (size_t)n_chunks * H;
  size_t off = 0;
  L.qg = off; off = align256(off + nh * kChunk * K * esize);
  L.kd = off; off = align256(off + nh * kChunk * K * esize);
  L.w = off; off = align256(off + nh * kChunk * K * esize);
  L.u = off; off = align256(off + nh * kChunk * V * esize);
  L.vn = off; off = align256(off + nh * kChunk * V * esize);
  L.aqk = off; off = align256(off + nh * kChunk * kChunk * esize);
  L.a = off; off = align256(off + nh * kChunk * kChunk * esize);
  L.gl = off; off = align256(off + nh * K * sizeof(float));
  L.h = off; off = align256(off + nh * (size_t)K * V * esize);
  L.total = off;
  return L;
}

// Backward workspace per (chunk, head):  dh : [K][V] (T)  gradient w.r.t. the
// state leaving the chunk;  dVN : [64][V] (T), stored transposed ([V][64]) by
// the bf16 tensor-core path, like VN;  for head sizes above 128 only, qk :
// [2][64][K] fp32, the pre-norm dq and dk rows (chunk_wide.cu).
struct BwdLayout {
  size_t dh, dvn, qk, total;
};

__host__ __device__ inline bool wide_heads(int K, int V) { return K > 128 || V > 128; }

__host__ __device__ inline BwdLayout bwd_layout(int64_t n_chunks, int H, int K, int V,
                                                int esize) {
  BwdLayout L;
  size_t nh = (size_t)n_chunks * H;
  size_t off = 0;
  L.dh = off; off = align256(off + nh * (size_t)K * V * esize);
  L.dvn = off; off = align256(off + nh * kChunk * V * esize);
  L.qk = off;
  if (wide_heads(K, V)) off = align256(off + nh * 2 * kChunk * (size_t)K * sizeof(float));
  L.total = off;
  return L;
}

}  // namespace gdn2
