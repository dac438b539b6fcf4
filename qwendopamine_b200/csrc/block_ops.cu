// block_ops.cu -- the GDN-2 block's prologue and epilogue around the core
// recurrence, and their extern "C" entry points:
//
// * causal depthwise convolution + SiLU over [B][T][D] token rows
//   (ShortConvolution, gdn2.py:372-430): forward, backward (dx, the prefix
//   gradient, and dweight / dbias through per-block partial sums reduced in a
//   fixed order), and the decode-cache update;
// * SiLU-gated RMSNorm over the last dimension (RMSNormGated,
//   gdn2.py:433-452), forward with the reference's input-dtype rounding after
//   every step, backward in fp32.
//
// Both are HBM-bound streaming kernels: each thread owns a few consecutive
// channels (one 8- or 16-byte vector of a row), a warp covers a contiguous
// run of a row's channels, and rows are loaded a run at a time before any
// arithmetic so every thread keeps several loads in flight.
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <type_traits>

#include "../../include/gdn2_b200.h"

#include "common.cuh"

namespace gdn2 {
int set_error(int code, const char* msg);  // abi.cu: the per-thread last error
namespace {

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return set_error(code, buf);
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(GDN2_ERR_CUDA, "%s: CUDA error %d (%s)", where, (int)e, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// 8-element vectors
// ---------------------------------------------------------------------------
// CPT consecutive elements of one row, moved as one 4-, 8-, 16- or 32-byte
// access (two 16-byte accesses for the last).
template <typename T, int CPT> struct Pack {
  static constexpr int kBytes = CPT * (int)sizeof(T);
  static_assert(kBytes == 4 || kBytes == 8 || kBytes % 16 == 0, "vector width");
  uint32_t u[kBytes / 4];
};

template <typename T, int CPT> __device__ __forceinline__ Pack<T, CPT> ldv(const T* p) {
  Pack<T, CPT> r;
  constexpr int nb = Pack<T, CPT>::kBytes;
  if constexpr (nb == 4) {
    r.u[0] = __ldg(reinterpret_cast<const unsigned int*>(p));
  } else if constexpr (nb == 8) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
    r.u[0] = v.x;
    r.u[1] = v.y;
  } else {
#pragma unroll
    for (int i = 0; i < nb / 16; ++i) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + i);
      r.u[4 * i] = v.x;
      r.u[4 * i + 1] = v.y;
      r.u[4 * i + 2] = v.z;
      r.u[4 * i + 3] = v.w;
    }
  }
  return r;
}

template <typename T, int CPT>
__device__ __forceinline__ void unpackv(const Pack<T, CPT>& r, float (&f)[CPT]) {
  const T* e = reinterpret_cast<const T*>(r.u);
#pragma unroll
  for (int i = 0; i < CPT; ++i) f[i] = to_f<T>(e[i]);
}

// Two fp32 values -> one 32-bit word of two 16-bit values (one packed
// round-to-nearest-even conversion).
template <typename T> __device__ __forceinline__ uint32_t pack_pair(float a, float b);
template <> __device__ __forceinline__ uint32_t pack_pair<__nv_bfloat16>(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <> __device__ __forceinline__ uint32_t pack_pair<__half>(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <typename T, int CPT> __device__ __forceinline__ void stv(T* p, const float (&f)[CPT]) {
  Pack<T, CPT> r;
  if constexpr (sizeof(T) == 2) {
#pragma unroll
    for (int i = 0; i < CPT / 2; ++i) r.u[i] = pack_pair<T>(f[2 * i], f[2 * i + 1]);
  } else {
    T* e = reinterpret_cast<T*>(r.u);
#pragma unroll
    for (int i = 0; i < CPT; ++i) e[i] = from_f<T>(f[i]);
  }
  constexpr int nb = Pack<T, CPT>::kBytes;
  if constexpr (nb == 4) {
    *reinterpret_cast<unsigned int*>(p) = r.u[0];
  } else if constexpr (nb == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(r.u[0], r.u[1]);
  } else {
#pragma unroll
    for (int i = 0; i < nb / 16; ++i)
      reinterpret_cast<uint4*>(p)[i] = make_uint4(r.u[4 * i], r.u[4 * i + 1], r.u[4 * i + 2],
                                                  r.u[4 * i + 3]);
  }
}

template <typename T, int CPT> __device__ __forceinline__ void zerov(Pack<T, CPT>& r) {
#pragma unroll
  for (int i = 0; i < Pack<T, CPT>::kBytes / 4; ++i) r.u[i] = 0u;
}

// Rounding to the token dtype (identity for fp32).
template <typename T> __device__ __forceinline__ float rnd(float x) { return to_f<T>(from_f<T>(x)); }

// Two values rounded at once: one packed conversion instead of two scalar
// ones (scalar float -> 16-bit conversions issue on the special-function
// pipe, which the SiLU's exponential and reciprocal already load).  Same
// round-to-nearest-even result per element.
template <typename T> __device__ __forceinline__ float2 rnd2(float2 v);
template <> __device__ __forceinline__ float2 rnd2<float>(float2 v) { return v; }
template <> __device__ __forceinline__ float2 rnd2<__nv_bfloat16>(float2 v) {
  return __bfloat1622float2(__floats2bfloat162_rn(v.x, v.y));
}
template <> __device__ __forceinline__ float2 rnd2<__half>(float2 v) {
  return __half22float2(__floats2half2_rn(v.x, v.y));
}

// SiLU in the reference's fp32 form x / (1 + exp(-x)), with the fast
// exponential and division intrinsics: a few fp32 ulps from the exact form,
// which after rounding to bf16 changed no output of the config-1 conv and
// norm forwards (the exact form cost 1.8x the conv forward's time).
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.f + __expf(-x)); }

__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.f, 1.f + __expf(-x)); }

// d silu / dx times dy, in the reference's fp32 form of the SiLU backward.
__device__ __forceinline__ float silu_bwd_f(float dy, float x) {
  const float s = sigmoid_f(x);
  return dy * s * (1.f + x * (1.f - s));
}

// ---------------------------------------------------------------------------
// causal depthwise convolution
// ---------------------------------------------------------------------------
constexpr int kConvStrip = 64;  // tokens per CTA (one strip of rows)
constexpr int kConvMaxW = 4;

struct ConvArgs {
  int B, T, D;
  const void* x;
  const float* w;     // [D][W]
  const float* bias;  // [D] or null
  const void* prefix;
  int64_t psb, psw, psd;
  void* y;
  void* new_state;    // [B][D][W-1] or null
  const void* dy;
  void* dx;
  float* part;        // [nblk][W+1][D]
  float* dprefix;     // [B][W-1][D] or null
  float* dweight;     // [D][W]
  float* dbias;       // [D] or null
  int seg;            // backward: rows per strip (grid.y strips per batch entry)
};

template <int W, int CPT>
__device__ __forceinline__ void load_weights(const ConvArgs& a, int d0, float (&wt)[W][CPT],
                                             float (&bs)[CPT]) {
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
#pragma unroll
    for (int j = 0; j < W; ++j) wt[j][i] = __ldg(a.w + (int64_t)(d0 + i) * W + j);
    bs[i] = a.bias ? __ldg(a.bias + d0 + i) : 0.f;
  }
}

// Row r (< 0 reads the prefix, row W-1+r of it) of batch entry b, channels d0..d0+CPT-1.
template <typename T, int W, int CPT>
__device__ __forceinline__ void load_row(const ConvArgs& a, const T* xb, int b, int d0, int r,
                                         float (&f)[CPT]) {
  if (r >= 0) {
    unpackv<T, CPT>(ldv<T, CPT>(xb + (int64_t)r * a.D), f);
  } else if (a.prefix) {
    const T* p = reinterpret_cast<const T*>(a.prefix) + b * a.psb + (W - 1 + r) * a.psw;
#pragma unroll
    for (int i = 0; i < CPT; ++i) f[i] = to_f<T>(p[(int64_t)(d0 + i) * a.psd]);
  } else {
#pragma unroll
    for (int i = 0; i < CPT; ++i) f[i] = 0.f;
  }
}

// Channels per thread: 4 (a warp covers 128 channels, 256 bytes of a bf16
// row; a CTA 1024 contiguous channels), which keeps the forward at 64
// registers (four CTAs per SM) and the backward under 128 (two), with the
// register window, the weights and a 4-row run in flight.
constexpr int kFwdCPT = 4;
constexpr int kBwdCPT = 4;
constexpr int kConvChannels = 256 * 4;  // channels per CTA (256 threads x 4)

// Channel pairs: the per-channel FMAs run as packed fp32x2 operations
// (__ffma2_rn and friends: two fp32 FMAs per instruction with the same
// rounding as fmaf, so the results equal the one-channel-at-a-time form).
template <int W, int CPT>
__device__ __forceinline__ void load_weight_pairs(const ConvArgs& a, int d0,
                                                  float2 (&wt)[W][CPT / 2], float2 (&bs)[CPT / 2]) {
  float w1[W][CPT], b1[CPT];
  load_weights<W, CPT>(a, d0, w1, b1);
#pragma unroll
  for (int p = 0; p < CPT / 2; ++p) {
#pragma unroll
    for (int j = 0; j < W; ++j) wt[j][p] = make_float2(w1[j][2 * p], w1[j][2 * p + 1]);
    bs[p] = make_float2(b1[2 * p], b1[2 * p + 1]);
  }
}

template <typename T, int W, int CPT>
__device__ __forceinline__ void load_row_pairs(const ConvArgs& a, const T* xb, int b, int d0,
                                               int r, float2 (&f2)[CPT / 2]) {
  float f[CPT];
  load_row<T, W, CPT>(a, xb, b, d0, r, f);
#pragma unroll
  for (int p = 0; p < CPT / 2; ++p) f2[p] = make_float2(f[2 * p], f[2 * p + 1]);
}

// y = act(round(bias + sum_j w_j x_{t-W+1+j})): grid (D/1024, T/64, B); a
// CTA walks a 64-token strip of 1024 contiguous channels (every row access of
// the CTA is 2 KB contiguous), each thread 4 channels, with the W-1 previous
// rows carried in registers.
template <typename T, int W, int ACT>
__global__ void __launch_bounds__(256, 2) k_conv_fwd(ConvArgs a) {
  constexpr int CPT = kFwdCPT, CP = CPT / 2;
  constexpr int R = 4;  // rows loaded per run
  constexpr int WP = W > 1 ? W - 1 : 1;
  const int d0 = (blockIdx.x * 256 + threadIdx.x) * CPT;
  const int b = blockIdx.z;
  const int tb = blockIdx.y * kConvStrip;
  if (d0 >= a.D) return;
  const int te = min(tb + kConvStrip, a.T);
  float2 wt[W][CP], bs[CP];
  load_weight_pairs<W, CPT>(a, d0, wt, bs);
  const T* xb = reinterpret_cast<const T*>(a.x) + (int64_t)b * a.T * a.D + d0;
  T* yb = reinterpret_cast<T*>(a.y) + (int64_t)b * a.T * a.D + d0;
  float2 win[WP][CP];
#pragma unroll
  for (int i = 0; i < W - 1; ++i)
    load_row_pairs<T, W, CPT>(a, xb, b, d0, tb - (W - 1) + i, win[i]);
  for (int t0 = tb; t0 < te; t0 += R) {
    Pack<T, CPT> raw[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (t0 + r < te) raw[r] = ldv<T, CPT>(xb + (int64_t)(t0 + r) * a.D);
      else zerov<T, CPT>(raw[r]);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (t0 + r >= te) continue;  // (predicated: the loop stays unrolled)
      float cur[CPT], o[CPT];
      unpackv<T, CPT>(raw[r], cur);
#pragma unroll
      for (int p = 0; p < CP; ++p) {
        const float2 c2 = make_float2(cur[2 * p], cur[2 * p + 1]);
        float2 acc = bs[p];
#pragma unroll
        for (int j = 0; j < W - 1; ++j) acc = __ffma2_rn(wt[j][p], win[j][p], acc);
        acc = __ffma2_rn(wt[W - 1][p], c2, acc);
        const float2 cr = rnd2<T>(acc);
        o[2 * p] = ACT ? silu_f(cr.x) : cr.x;
        o[2 * p + 1] = ACT ? silu_f(cr.y) : cr.y;
#pragma unroll
        for (int j = 0; j + 1 < W - 1; ++j) win[j][p] = win[j + 1][p];
        if (W > 1) win[WP - 1][p] = c2;
      }
      stv<T, CPT>(yb + (int64_t)(t0 + r) * a.D, o);
    }
  }
  // the strip holding the last row leaves rows T-W+1 .. T-1 in its window
  if (a.new_state && te == a.T && W > 1) {
    T* ns = reinterpret_cast<T*>(a.new_state) + ((int64_t)b * a.D + d0) * (W - 1);
#pragma unroll
    for (int p = 0; p < CP; ++p)
#pragma unroll
      for (int j = 0; j < W - 1; ++j) {
        ns[(2 * p) * (W - 1) + j] = from_f<T>(win[j][p].x);
        ns[(2 * p + 1) * (W - 1) + j] = from_f<T>(win[j][p].y);
      }
  }
}

// One row of the backward (see k_conv_bwd): dc_s from dy_s and the
// recomputed pre-activation, the dweight / dbias partial sums, and dx_t for
// t = s - W + 1 out of the W-1 previous dc values.  EDGE = false is the
// strip interior (s < T, s < te, tb <= t < te), where every test drops out.
template <typename T, int W, int ACT, bool EDGE>
__device__ __forceinline__ void conv_bwd_row(const ConvArgs& a, int s, int tb, int te, int send,
                                             bool want_dprefix, int b, int d0,
                                             const Pack<T, kBwdCPT>& rx,
                                             const Pack<T, kBwdCPT>& rdy,
                                             const float2 (&wt)[W][kBwdCPT / 2],
                                             const float2 (&bs)[kBwdCPT / 2],
                                             float2 (&win)[W > 1 ? W - 1 : 1][kBwdCPT / 2],
                                             float2 (&dcw)[W > 1 ? W - 1 : 1][kBwdCPT / 2],
                                             float2 (&dwp)[W + 1][kBwdCPT / 2], T* dxb) {
  constexpr int CPT = kBwdCPT, CP = CPT / 2, WP = W > 1 ? W - 1 : 1;
  if (EDGE && s >= send) return;
  float cur[CPT], dy[CPT], o[CPT];
  unpackv<T, CPT>(rx, cur);
  unpackv<T, CPT>(rdy, dy);
  const int t = s - (W - 1);  // the input row emitted at this step
#pragma unroll
  for (int p = 0; p < CP; ++p) {
    const float2 c2 = make_float2(cur[2 * p], cur[2 * p + 1]);
    float2 dc = make_float2(0.f, 0.f);
    if (!EDGE || s < a.T) {
      dc = make_float2(dy[2 * p], dy[2 * p + 1]);
      if (ACT) {
        float2 acc = bs[p];
#pragma unroll
        for (int j = 0; j < W - 1; ++j) acc = __ffma2_rn(wt[j][p], win[j][p], acc);
        acc = __ffma2_rn(wt[W - 1][p], c2, acc);
        const float2 cr = rnd2<T>(acc);
        dc = rnd2<T>(make_float2(silu_bwd_f(dc.x, cr.x), silu_bwd_f(dc.y, cr.y)));
      }
      if (!EDGE || s < te) {
#pragma unroll
        for (int j = 0; j < W - 1; ++j) dwp[j][p] = __ffma2_rn(dc, win[j][p], dwp[j][p]);
        dwp[W - 1][p] = __ffma2_rn(dc, c2, dwp[W - 1][p]);
        dwp[W][p] = __fadd2_rn(dwp[W][p], dc);
      }
    }
    float2 acc = __fmul2_rn(wt[0][p], dc);
#pragma unroll
    for (int j = 1; j < W; ++j) acc = __ffma2_rn(wt[j][p], dcw[W - 1 - j][p], acc);
    o[2 * p] = acc.x;
    o[2 * p + 1] = acc.y;
#pragma unroll
    for (int j = 0; j + 1 < W - 1; ++j) {
      win[j][p] = win[j + 1][p];
      dcw[j][p] = dcw[j + 1][p];
    }
    if (W > 1) {
      win[WP - 1][p] = c2;
      dcw[WP - 1][p] = dc;
    }
  }
  if (!EDGE) {
    stv<T, CPT>(dxb + (int64_t)t * a.D, o);
  } else if (t >= tb) {
    if (t < te) stv<T, CPT>(dxb + (int64_t)t * a.D, o);
  } else if (want_dprefix && t >= -(W - 1)) {
    float* dp = a.dprefix + ((int64_t)b * (W - 1) + (t + W - 1)) * a.D + d0;
#pragma unroll
    for (int i = 0; i < CPT; ++i) dp[i] = o[i];
  }
}

// x and dy rows s0 .. s0+R-1 (zeros past T or past the strip's last row).
template <typename T, int R>
__device__ __forceinline__ void conv_bwd_loads(const ConvArgs& a, const T* xb, const T* dyb,
                                               int s0, int send, Pack<T, kBwdCPT> (&rx)[R],
                                               Pack<T, kBwdCPT> (&rdy)[R]) {
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int s = s0 + r;
    if (s < a.T && s < send) {
      rx[r] = ldv<T, kBwdCPT>(xb + (int64_t)s * a.D);
      rdy[r] = ldv<T, kBwdCPT>(dyb + (int64_t)s * a.D);
    } else {
      zerov<T, kBwdCPT>(rx[r]);
      zerov<T, kBwdCPT>(rdy[r]);
    }
  }
}

// Backward over the strip's rows s in [tb, te + W - 1) (strip = a.seg rows):
// dc_s = act'(c_s) dy_s (rounded to the token dtype, as the reference's
// activation backward is), dx_t = sum_j w_j dc_{t+W-1-j} emitted at
// s = t + W - 1, dw_j += dc_s x_{s-W+1+j} and dbias += dc_s for s < te.
// Rows t < 0 of the first strip are the prefix rows (dprefix).  Rows go R at
// a time, the next R rows' loads issued before this run's arithmetic (two
// runs in flight per thread).  Each thread's sums of dw / dbias for its
// channels go to part[blk][j][d] (blk = the CTA's strip), reduced over the
// strips in a fixed order by k_col_sum.
template <typename T, int W, int ACT>
__global__ void __launch_bounds__(256, 2) k_conv_bwd(ConvArgs a) {
  constexpr int CPT = kBwdCPT, CP = CPT / 2;
  constexpr int R = sizeof(T) == 4 ? 2 : 4;  // (fp32 rows are twice as many registers)
  constexpr int WP = W > 1 ? W - 1 : 1;
  const int d0 = (blockIdx.x * 256 + threadIdx.x) * CPT;
  const int b = blockIdx.z;
  const int tb = blockIdx.y * a.seg;
  if (d0 >= a.D) return;
  float2 dwp[W + 1][CP];
#pragma unroll
  for (int j = 0; j <= W; ++j)
#pragma unroll
    for (int p = 0; p < CP; ++p) dwp[j][p] = make_float2(0.f, 0.f);
  const int te = min(tb + a.seg, a.T);
  float2 wt[W][CP], bs[CP];
  load_weight_pairs<W, CPT>(a, d0, wt, bs);
  const T* xb = reinterpret_cast<const T*>(a.x) + (int64_t)b * a.T * a.D + d0;
  const T* dyb = reinterpret_cast<const T*>(a.dy) + (int64_t)b * a.T * a.D + d0;
  T* dxb = reinterpret_cast<T*>(a.dx) + (int64_t)b * a.T * a.D + d0;
  float2 win[WP][CP], dcw[WP][CP];  // previous W-1 input rows and dc values
#pragma unroll
  for (int i = 0; i < W - 1; ++i) {
    load_row_pairs<T, W, CPT>(a, xb, b, d0, tb - (W - 1) + i, win[i]);
#pragma unroll
    for (int p = 0; p < CP; ++p) dcw[i][p] = make_float2(0.f, 0.f);
  }
  const int send = te + W - 1;
  const bool want_dprefix = a.dprefix && tb == 0;
  Pack<T, CPT> rx[R], rdy[R];
  conv_bwd_loads<T, R>(a, xb, dyb, tb, send, rx, rdy);
  for (int s0 = tb; s0 < send; s0 += R) {
    Pack<T, CPT> nx[R], ndy[R];
    if (s0 + R < send) conv_bwd_loads<T, R>(a, xb, dyb, s0 + R, send, nx, ndy);
    if (s0 >= tb + W - 1 && s0 + R <= te) {
#pragma unroll
      for (int r = 0; r < R; ++r)
        conv_bwd_row<T, W, ACT, false>(a, s0 + r, tb, te, send, want_dprefix, b, d0, rx[r],
                                       rdy[r], wt, bs, win, dcw, dwp, dxb);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r)
        conv_bwd_row<T, W, ACT, true>(a, s0 + r, tb, te, send, want_dprefix, b, d0, rx[r],
                                      rdy[r], wt, bs, win, dcw, dwp, dxb);
    }
#pragma unroll
    for (int r = 0; r < R; ++r) {
      rx[r] = nx[r];
      rdy[r] = ndy[r];
    }
  }
  const int blk = blockIdx.z * gridDim.y + blockIdx.y;
#pragma unroll
  for (int j = 0; j <= W; ++j) {
    float* pp = a.part + ((int64_t)blk * (W + 1) + j) * a.D + d0;
#pragma unroll
    for (int p = 0; p < CP; ++p) {
      pp[2 * p] = dwp[j][p].x;
      pp[2 * p + 1] = dwp[j][p].y;
    }
  }
}

// Column sums of part[nblk][ncol] in a fixed order: a CTA takes 32 columns;
// its 8 warps take the rows k = g, g + 8, ... (four loads in flight each) and
// the 8 partial sums are added in warp order.  The sum of column col goes to
// out[col] (W == 0), or, for the convolution's [W+1][D] partials, to
// dweight[d][j] (col = j D + d, j < W) and dbias[d] (j = W).
__global__ void __launch_bounds__(256) k_col_sum(const float* part, int nblk, int ncol, int W,
                                                 int D, float* out, float* dbias) {
  __shared__ float red[8][32];
  const int lane = threadIdx.x & 31, g = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (col < ncol) {
    int k = g;
    for (; k + 24 < nblk; k += 32) {
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += part[(int64_t)(k + 8 * u) * ncol + col];
    }
    for (; k < nblk; k += 8) acc[0] += part[(int64_t)k * ncol + col];
  }
  red[g][lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  if (g == 0 && col < ncol) {
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum += red[i][lane];
    if (W == 0) {
      out[col] = sum;
    } else {
      const int j = col / D, d = col - j * D;
      if (j < W) out[(int64_t)d * W + j] = sum;
      else if (dbias) dbias[d] = sum;
    }
  }
}

// Upper bound of the backward's strip count (the partial-sum rows): never
// more than ceil(T / kConvStrip) strips per batch entry.
int conv_nblk(const gdn2_conv_problem* p) {
  return p->B * ((p->T + kConvStrip - 1) / kConvStrip);
}

// Backward strips: one wave.  With `slots` CTAs resident on the GPU and
// B x ceil(D / 1024) channel columns, each column of T rows is cut into
// floor(slots / columns) strips (at least one, at most ceil(T / kConvStrip)),
// so every SM gets the same number of rows and no CTA waits for a second
// wave; many columns (more than the slots) fall back to one strip each.
template <typename K>
cudaError_t conv_bwd_strip(K kernel, const gdn2_conv_problem* p, int* seg) {
  int sms = 0, occ = 0;
  cudaError_t e = num_sms(&sms);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, 256, 0);
  if (e != cudaSuccess) return e;
  const int64_t cols = (int64_t)p->B * ((p->D + kConvChannels - 1) / kConvChannels);
  const int64_t slots = (int64_t)sms * (occ > 0 ? occ : 1);
  const int64_t most = (p->T + kConvStrip - 1) / kConvStrip;
  int64_t n = slots / cols;
  n = n < 1 ? 1 : (n > most ? most : n);
  *seg = (int)((p->T + n - 1) / n);
  return cudaSuccess;
}

template <typename T, int W>
cudaError_t launch_conv(const gdn2_conv_problem* p, const ConvArgs& a0, bool bwd,
                        cudaStream_t st) {
  static_assert(kFwdCPT * 256 == kConvChannels && kBwdCPT * 256 == kConvChannels, "CTA width");
  const int gx = (p->D + kConvChannels - 1) / kConvChannels;
  if (!bwd) {
    dim3 grid(gx, (p->T + kConvStrip - 1) / kConvStrip, p->B);
    if (p->activation) k_conv_fwd<T, W, 1><<<grid, 256, 0, st>>>(a0);
    else k_conv_fwd<T, W, 0><<<grid, 256, 0, st>>>(a0);
    return cudaGetLastError();
  }
  ConvArgs a = a0;
  auto kern = p->activation ? k_conv_bwd<T, W, 1> : k_conv_bwd<T, W, 0>;
  cudaError_t e = conv_bwd_strip(kern, p, &a.seg);
  if (e != cudaSuccess) return e;
  const int nseg = (p->T + a.seg - 1) / a.seg;
  kern<<<dim3(gx, nseg, p->B), 256, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int n = (W + 1) * p->D;
  k_col_sum<<<(n + 31) / 32, 256, 0, st>>>(a.part, p->B * nseg, n, W, p->D, a.dweight, a.dbias);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// SiLU-gated RMSNorm
// ---------------------------------------------------------------------------
constexpr int kNormMaxBlocks = 1024;
constexpr int kNormUnroll = 1;  // row groups loaded per trip (2 measured slower)

struct NormArgs {
  int64_t rows;
  int N;
  float eps;
  const void* x;
  const void* z;
  const void* w;
  void* y;
  const void* dy;
  void* dx;
  void* dz;
  float* part;     // [nblk][N]
  float* dweight;  // [N]
};

// TPR threads per row, 8 columns each (col = 8 * (v * TPR + sub)); the row's
// sums are reduced over the TPR lanes with shuffles.
template <int TPR> __device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename TW> __device__ __forceinline__ void load_w8(const TW* w, int c, int N,
                                                             float (&f)[8]) {
  if (c < N) {
    unpackv<TW, 8>(ldv<TW, 8>(w + c), f);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = 0.f;
  }
}

// Forward, in the reference's order and input-dtype rounding:
//   var = round(mean(round(x^2))), r = round(rsqrt(round(var + eps))),
//   n = round(x r), n = round(n w) (or n w in fp32 for an fp32 weight),
//   y = round_out(n round(silu(z))).
// F32 (the reference under autocast): the same steps without rounding,
// except silu(z), which runs in the input dtype.
template <typename T, typename TW, typename TO, int TPR, bool F32, int EPT>
__global__ void __launch_bounds__(256) k_gnorm_fwd(NormArgs a) {
  // EPT columns per lane (8, or 16 when the row is exactly 16 TPR wide: half
  // the lanes per row, so half the shuffles)
  constexpr int RPC = 256 / TPR, U = kNormUnroll, NP = EPT / 8;
  static_assert(EPT == 8 || EPT == 16, "8 or 16 columns per lane");
  const int sub = threadIdx.x % TPR, slot = threadIdx.x / TPR;
  const int c = EPT * sub;
  const bool live = c < a.N;
  float w[NP][8];
#pragma unroll
  for (int p = 0; p < NP; ++p) load_w8<TW>(reinterpret_cast<const TW*>(a.w), c + 8 * p, a.N, w[p]);
  const float inv_n = 1.f / (float)a.N;
  // The trip count is uniform across the CTA: a row's lanes share a warp
  // with other rows' lanes, and every lane joins the shuffles of each trip.
  // Each trip loads U row groups before any arithmetic.
  for (int64_t base = (int64_t)blockIdx.x * RPC * U; base < a.rows;
       base += (int64_t)gridDim.x * RPC * U) {
    Pack<T, 8> px[U][NP], pz[U][NP];
    bool on[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = base + u * RPC + slot;
      on[u] = live && row < a.rows;
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        if (on[u]) {
          px[u][p] = ldv<T, 8>(reinterpret_cast<const T*>(a.x) + row * a.N + c + 8 * p);
          pz[u][p] = ldv<T, 8>(reinterpret_cast<const T*>(a.z) + row * a.N + c + 8 * p);
        } else {
          zerov<T, 8>(px[u][p]);
          zerov<T, 8>(pz[u][p]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float x[NP][8], z[NP][8];
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        unpackv<T, 8>(px[u][p], x[p]);
        unpackv<T, 8>(pz[u][p], z[p]);
      }
      using TR = typename std::conditional<F32, float, T>::type;  // intermediate rounding
      float ss = 0.f;
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float2 sq = rnd2<TR>(make_float2(x[p][i] * x[p][i], x[p][i + 1] * x[p][i + 1]));
          ss += sq.x;
          ss += sq.y;
        }
      ss = group_sum<TPR>(ss);
      const float var = rnd<TR>(ss * inv_n);
      const float r = rnd<TR>(rsqrtf(rnd<TR>(var + a.eps)));
#pragma unroll
      for (int p = 0; p < NP; ++p) {
        using TN = typename std::conditional<F32, float, TW>::type;  // the n * w rounding
        float y[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float2 n = rnd2<TR>(make_float2(x[p][i] * r, x[p][i + 1] * r));
          n = rnd2<TN>(make_float2(n.x * w[p][i], n.y * w[p][i + 1]));
          const float2 s = rnd2<T>(make_float2(silu_f(z[p][i]), silu_f(z[p][i + 1])));
          y[i] = n.x * s.x;
          y[i + 1] = n.y * s.y;
        }
        if (on[u])
          stv<TO, 8>(reinterpret_cast<TO*>(a.y) + (base + u * RPC + slot) * a.N + c + 8 * p, y);
      }
    }
  }
}

// Backward in fp32: r = rsqrt(mean(x^2) + eps), n = x r, s = silu(z),
//   dn = dy w s, dx = r (dn - n mean(dn n)), dz = dy n w silu'(z),
//   dweight = sum_rows dy n s (per-CTA partials, reduced in a fixed order).
template <typename T, typename TW, typename TO, int TPR>
__global__ void __launch_bounds__(256) k_gnorm_bwd(NormArgs a) {
  constexpr int RPC = 256 / TPR, U = kNormUnroll;
  __shared__ float red[256 * 8];
  const int sub = threadIdx.x % TPR, slot = threadIdx.x / TPR;
  const int c = 8 * sub;
  const bool live = c < a.N;
  float w[8], dwp[8];
  load_w8<TW>(reinterpret_cast<const TW*>(a.w), c, a.N, w);
#pragma unroll
  for (int i = 0; i < 8; ++i) dwp[i] = 0.f;
  const float inv_n = 1.f / (float)a.N;
  // CTA-uniform trip count and U row groups loaded per trip (see the forward)
  for (int64_t base = (int64_t)blockIdx.x * RPC * U; base < a.rows;
       base += (int64_t)gridDim.x * RPC * U) {
    Pack<T, 8> px[U], pz[U];
    Pack<TO, 8> pd[U];
    bool on[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t row = base + u * RPC + slot;
      on[u] = live && row < a.rows;
      if (on[u]) {
        px[u] = ldv<T, 8>(reinterpret_cast<const T*>(a.x) + row * a.N + c);
        pz[u] = ldv<T, 8>(reinterpret_cast<const T*>(a.z) + row * a.N + c);
        pd[u] = ldv<TO, 8>(reinterpret_cast<const TO*>(a.dy) + row * a.N + c);
      } else {
        zerov<T, 8>(px[u]);
        zerov<T, 8>(pz[u]);
        zerov<TO, 8>(pd[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float x[8], z[8], dy[8];
      unpackv<T, 8>(px[u], x);
      unpackv<T, 8>(pz[u], z);
      unpackv<TO, 8>(pd[u], dy);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
      ss = group_sum<TPR>(ss);
      const float r = rsqrtf(ss * inv_n + a.eps);
      float n[8], dn[8], dz[8], dot = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float sg = sigmoid_f(z[i]);
        const float s = z[i] * sg;
        n[i] = x[i] * r;
        dn[i] = dy[i] * w[i] * s;
        dot = fmaf(dn[i], n[i], dot);
        dz[i] = dy[i] * n[i] * w[i] * sg * (1.f + z[i] * (1.f - sg));
        dwp[i] = fmaf(dy[i] * n[i], s, dwp[i]);
      }
      dot = group_sum<TPR>(dot) * inv_n;
      float dx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) dx[i] = r * (dn[i] - n[i] * dot);
      if (on[u]) {
        const int64_t row = base + u * RPC + slot;
        stv<T, 8>(reinterpret_cast<T*>(a.dx) + row * a.N + c, dx);
        stv<T, 8>(reinterpret_cast<T*>(a.dz) + row * a.N + c, dz);
      }
    }
  }
  // CTA sum over the RPC row slots, column by column in a fixed order
#pragma unroll
  for (int i = 0; i < 8; ++i) red[slot * (TPR * 8) + c + i] = dwp[i];
  __syncthreads();
  for (int col = threadIdx.x; col < TPR * 8; col += 256) {
    float sum = 0.f;
    for (int k = 0; k < RPC; ++k) sum += red[k * (TPR * 8) + col];
    if (col < a.N) a.part[(int64_t)blockIdx.x * a.N + col] = sum;
  }
}

int norm_tpr(int N) {
  if (N % 8 != 0 || N <= 0 || N > 256) return 0;
  return N <= 64 ? 8 : (N <= 128 ? 16 : 32);
}

// Upper bound of the CTA count (the backward's partial-sum rows).
int norm_nblk(const gdn2_norm_problem* p) {
  const int per = 256 / norm_tpr(p->N) * kNormUnroll;
  const int64_t need = (p->rows + per - 1) / per;
  return (int)(need < kNormMaxBlocks ? need : kNormMaxBlocks);
}

// CTAs actually launched: no more than fit on the GPU at once, so the
// row-group loop has no partial last wave.
template <typename K>
cudaError_t norm_grid(K kernel, const gdn2_norm_problem* p, int* grid) {
  int sms = 0, occ = 0;
  cudaError_t e = num_sms(&sms);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, 256, 0);
  if (e != cudaSuccess) return e;
  const int cap = sms * (occ > 0 ? occ : 1), ub = norm_nblk(p);
  *grid = ub < cap ? ub : cap;
  return cudaSuccess;
}

template <typename T, typename TW, typename TO, int TPR>
cudaError_t launch_gnorm2(const gdn2_norm_problem* p, const NormArgs& a, bool bwd,
                          cudaStream_t st) {
  int nblk = 0;
  cudaError_t e;
  if (!bwd) {
    auto k = p->fp32_math ? k_gnorm_fwd<T, TW, TO, TPR, true, 8>
                          : k_gnorm_fwd<T, TW, TO, TPR, false, 8>;
    if ((e = norm_grid(k, p, &nblk)) != cudaSuccess) return e;
    k<<<nblk, 256, 0, st>>>(a);
    return cudaGetLastError();
  }
  if ((e = norm_grid(k_gnorm_bwd<T, TW, TO, TPR>, p, &nblk)) != cudaSuccess) return e;
  k_gnorm_bwd<T, TW, TO, TPR><<<nblk, 256, 0, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_col_sum<<<(p->N + 31) / 32, 256, 0, st>>>(a.part, nblk, p->N, 0, 0, a.dweight, nullptr);
  return cudaGetLastError();
}

// Forward over rows of 16 TPR columns, 16 per lane.
template <typename T, typename TW, typename TO, int TPR>
cudaError_t launch_gnorm_fwd16(const gdn2_norm_problem* p, const NormArgs& a, cudaStream_t st) {
  auto k = p->fp32_math ? k_gnorm_fwd<T, TW, TO, TPR, true, 16>
                        : k_gnorm_fwd<T, TW, TO, TPR, false, 16>;
  int nblk = 0;
  const cudaError_t e = norm_grid(k, p, &nblk);
  if (e != cudaSuccess) return e;
  k<<<nblk, 256, 0, st>>>(a);
  return cudaGetLastError();
}

template <typename T, typename TW, typename TO>
cudaError_t launch_gnorm(const gdn2_norm_problem* p, const NormArgs& a, bool bwd, cudaStream_t st) {
  if (!bwd && p->N == 128) return launch_gnorm_fwd16<T, TW, TO, 8>(p, a, st);
  if (!bwd && p->N == 256) return launch_gnorm_fwd16<T, TW, TO, 16>(p, a, st);
  switch (norm_tpr(p->N)) {
    case 8: return launch_gnorm2<T, TW, TO, 8>(p, a, bwd, st);
    case 16: return launch_gnorm2<T, TW, TO, 16>(p, a, bwd, st);
    default: return launch_gnorm2<T, TW, TO, 32>(p, a, bwd, st);
  }
}

// ---------------------------------------------------------------------------
// entry-point helpers
// ---------------------------------------------------------------------------
bool dtype_valid(int dt) {
  return dt == GDN2_DTYPE_F32 || dt == GDN2_DTYPE_BF16 || dt == GDN2_DTYPE_F16;
}

bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int check_conv(const gdn2_conv_problem* p, const char* fn) {
  if (!p) return fail(GDN2_ERR_INVALID, "%s: null problem", fn);
  if (p->B <= 0 || p->T <= 0 || p->D <= 0 || p->W <= 0)
    return fail(GDN2_ERR_INVALID, "%s: B, T, D, W must be positive (got %d, %d, %d, %d)", fn,
                p->B, p->T, p->D, p->W);
  if (!dtype_valid(p->dtype)) return fail(GDN2_ERR_INVALID, "%s: bad dtype %d", fn, p->dtype);
  if (p->activation != 0 && p->activation != 1)
    return fail(GDN2_ERR_INVALID, "%s: activation must be 0 or 1", fn);
  if (p->W > kConvMaxW || p->D % 8 != 0)
    return fail(GDN2_ERR_UNSUPPORTED, "%s: needs W <= %d and D %% 8 == 0 (W=%d, D=%d)", fn,
                kConvMaxW, p->W, p->D);
  return GDN2_OK;
}

template <typename T>
cudaError_t conv_dispatch_w(const gdn2_conv_problem* p, const ConvArgs& a, bool bwd,
                            cudaStream_t st) {
  switch (p->W) {
    case 1: return launch_conv<T, 1>(p, a, bwd, st);
    case 2: return launch_conv<T, 2>(p, a, bwd, st);
    case 3: return launch_conv<T, 3>(p, a, bwd, st);
    default: return launch_conv<T, 4>(p, a, bwd, st);
  }
}

cudaError_t conv_dispatch(const gdn2_conv_problem* p, const ConvArgs& a, bool bwd,
                          cudaStream_t st) {
  switch (p->dtype) {
    case GDN2_DTYPE_F32: return conv_dispatch_w<float>(p, a, bwd, st);
    case GDN2_DTYPE_BF16: return conv_dispatch_w<__nv_bfloat16>(p, a, bwd, st);
    default: return conv_dispatch_w<__half>(p, a, bwd, st);
  }
}

int check_norm(const gdn2_norm_problem* p, const char* fn) {
  if (!p) return fail(GDN2_ERR_INVALID, "%s: null problem", fn);
  if (p->rows < 0 || p->N <= 0)
    return fail(GDN2_ERR_INVALID, "%s: rows >= 0 and N > 0 required", fn);
  if (!dtype_valid(p->dtype) || !dtype_valid(p->weight_dtype))
    return fail(GDN2_ERR_INVALID, "%s: bad dtype", fn);
  if (p->weight_dtype != p->dtype && p->weight_dtype != GDN2_DTYPE_F32)
    return fail(GDN2_ERR_UNSUPPORTED, "%s: weight dtype must be the input dtype or fp32", fn);
  if (p->fp32_math != 0 && p->fp32_math != 1)
    return fail(GDN2_ERR_INVALID, "%s: fp32_math must be 0 or 1", fn);
  if (p->fp32_math && p->weight_dtype != GDN2_DTYPE_F32)
    return fail(GDN2_ERR_INVALID, "%s: fp32_math needs an fp32 weight", fn);
  if (!norm_tpr(p->N))
    return fail(GDN2_ERR_UNSUPPORTED, "%s: N %% 8 == 0 and N <= 256 required (N=%d)", fn, p->N);
  return GDN2_OK;
}

cudaError_t norm_dispatch(const gdn2_norm_problem* p, const NormArgs& a, bool bwd,
                          cudaStream_t st) {
  const bool wf = p->weight_dtype == GDN2_DTYPE_F32;
  switch (p->dtype) {
    case GDN2_DTYPE_F32: return launch_gnorm<float, float, float>(p, a, bwd, st);
    case GDN2_DTYPE_BF16:
      return wf ? launch_gnorm<__nv_bfloat16, float, float>(p, a, bwd, st)
                : launch_gnorm<__nv_bfloat16, __nv_bfloat16, __nv_bfloat16>(p, a, bwd, st);
    default:
      return wf ? launch_gnorm<__half, float, float>(p, a, bwd, st)
                : launch_gnorm<__half, __half, __half>(p, a, bwd, st);
  }
}

}  // namespace
}  // namespace gdn2

using namespace gdn2;

extern "C" {

int gdn2_conv_fwd(const gdn2_conv_problem* p, const void* x, const float* weight,
                  const float* bias, const void* prefix, void* y, void* new_state,
                  void* stream) {
  int rc = check_conv(p, "gdn2_conv_fwd");
  if (rc) return rc;
  if (!x || !weight || !y) return fail(GDN2_ERR_INVALID, "gdn2_conv_fwd: null pointer");
  if (!al16(x) || !al16(y))
    return fail(GDN2_ERR_INVALID, "gdn2_conv_fwd: x and y must start on a 16-byte boundary");
  ConvArgs a{};
  a.B = p->B; a.T = p->T; a.D = p->D;
  a.x = x; a.w = weight; a.bias = bias; a.prefix = prefix;
  a.psb = p->prefix_sb; a.psw = p->prefix_sw; a.psd = p->prefix_sd;
  a.y = y; a.new_state = new_state;
  cudaError_t e = conv_dispatch(p, a, false, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_conv_fwd");
}

size_t gdn2_conv_bwd_workspace_bytes(const gdn2_conv_problem* p) {
  if (check_conv(p, "gdn2_conv_bwd_workspace_bytes") != GDN2_OK) return 0;
  return (size_t)conv_nblk(p) * (p->W + 1) * p->D * sizeof(float);
}

int gdn2_conv_bwd(const gdn2_conv_problem* p, const void* x, const float* weight,
                  const float* bias, const void* prefix, const void* dy, void* dx,
                  float* dweight, float* dbias, float* dprefix, void* workspace,
                  size_t workspace_bytes, void* stream) {
  int rc = check_conv(p, "gdn2_conv_bwd");
  if (rc) return rc;
  if (!x || !weight || !dy || !dx || !dweight || !workspace)
    return fail(GDN2_ERR_INVALID, "gdn2_conv_bwd: null pointer");
  if (!al16(x) || !al16(dy) || !al16(dx))
    return fail(GDN2_ERR_INVALID, "gdn2_conv_bwd: x, dy, dx must start on a 16-byte boundary");
  const size_t need = gdn2_conv_bwd_workspace_bytes(p);
  if (workspace_bytes < need)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_conv_bwd: workspace %zu < %zu bytes", workspace_bytes,
                need);
  ConvArgs a{};
  a.B = p->B; a.T = p->T; a.D = p->D;
  a.x = x; a.w = weight; a.bias = bias; a.prefix = prefix;
  a.psb = p->prefix_sb; a.psw = p->prefix_sw; a.psd = p->prefix_sd;
  a.dy = dy; a.dx = dx; a.part = static_cast<float*>(workspace);
  a.dprefix = dprefix; a.dweight = dweight; a.dbias = dbias;
  cudaError_t e = conv_dispatch(p, a, true, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_conv_bwd");
}

int gdn2_gated_norm_fwd(const gdn2_norm_problem* p, const void* x, const void* z,
                        const void* weight, void* y, void* stream) {
  int rc = check_norm(p, "gdn2_gated_norm_fwd");
  if (rc) return rc;
  if (p->rows == 0) return GDN2_OK;
  if (!x || !z || !weight || !y) return fail(GDN2_ERR_INVALID, "gdn2_gated_norm_fwd: null pointer");
  if (!al16(x) || !al16(z) || !al16(weight) || !al16(y))
    return fail(GDN2_ERR_INVALID, "gdn2_gated_norm_fwd: tensors must start on a 16-byte boundary");
  NormArgs a{};
  a.rows = p->rows; a.N = p->N; a.eps = p->eps;
  a.x = x; a.z = z; a.w = weight; a.y = y;
  cudaError_t e = norm_dispatch(p, a, false, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_gated_norm_fwd");
}

size_t gdn2_gated_norm_bwd_workspace_bytes(const gdn2_norm_problem* p) {
  if (check_norm(p, "gdn2_gated_norm_bwd_workspace_bytes") != GDN2_OK) return 0;
  return (size_t)(norm_nblk(p) > 0 ? norm_nblk(p) : 1) * p->N * sizeof(float);
}

int gdn2_gated_norm_bwd(const gdn2_norm_problem* p, const void* x, const void* z,
                        const void* weight, const void* dy, void* dx, void* dz,
                        float* dweight, void* workspace, size_t workspace_bytes,
                        void* stream) {
  int rc = check_norm(p, "gdn2_gated_norm_bwd");
  if (rc) return rc;
  if (!dweight) return fail(GDN2_ERR_INVALID, "gdn2_gated_norm_bwd: null dweight");
  if (p->rows == 0) {
    cudaError_t e = cudaMemsetAsync(dweight, 0, (size_t)p->N * sizeof(float), (cudaStream_t)stream);
    return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_gated_norm_bwd");
  }
  if (!x || !z || !weight || !dy || !dx || !dz || !workspace)
    return fail(GDN2_ERR_INVALID, "gdn2_gated_norm_bwd: null pointer");
  if (!al16(x) || !al16(z) || !al16(weight) || !al16(dy) || !al16(dx) || !al16(dz))
    return fail(GDN2_ERR_INVALID, "gdn2_gated_norm_bwd: tensors must start on a 16-byte boundary");
  const size_t need = gdn2_gated_norm_bwd_workspace_bytes(p);
  if (workspace_bytes < need)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_gated_norm_bwd: workspace %zu < %zu bytes",
                workspace_bytes, need);
  NormArgs a{};
  a.rows = p->rows; a.N = p->N; a.eps = p->eps;
  a.x = x; a.z = z; a.w = weight; a.dy = dy; a.dx = dx; a.dz = dz;
  a.part = static_cast<float*>(workspace); a.dweight = dweight;
  cudaError_t e = norm_dispatch(p, a, true, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_gated_norm_bwd");
}

}  // extern "C"
