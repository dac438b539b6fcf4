// recurrent.cu -- token-serial GDN-2 forward (decode / short prefill) on B200.
//
// Replaces the Triton kernel fused_recurrent_gdn2_fwd_kernel
// (fused_recurrent_gdn2.py:117-341).  The fp32 state is read once and written
// once per call with 128-bit streaming accesses -- the HBM floor of a decode
// step -- and stays in registers across the call's tokens.
// Per token:
//   S <- Diag(e^g) S;  r = S^T (b*k);  d = w*v - r;  S <- S + k d^T;  o = S^T q
// with q, k L2-normalised in kernel (x / sqrt(sum x^2 + 1e-6), as the Triton
// kernel does at :252-254) and q scaled after normalisation.
#include "chunk_args.cuh"

namespace gdn2 {

// One CTA per (sequence, value head, VB-column slice of the state): the
// slice's K x VB fp32 block lives in registers, thread (rg, cg) holding rows
// [rg*RPT, rg*RPT+RPT) x columns [4cg, 4cg+4) of the slice, so a warp moves
// two 256-byte row segments per 128-bit access.  Splitting the value columns
// keeps the per-thread state at 32 floats, which lets several CTAs share an
// SM and overlap one CTA's state load with another's store.
template <typename T, int D, int VB>
__global__ void __launch_bounds__(kThreads, 3) k_recurrent(RecArgs a) {
  constexpr int CG = VB / 4;           // column groups of 4 floats
  constexpr int RG = kThreads / CG;    // row groups
  constexpr int RPT = D / RG;          // state rows per thread
  __shared__ float sq[D], sk[D], sg[D], sb[D], sv[VB], sw[VB];
  __shared__ float red[RG][VB];
  __shared__ float snorm[2];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, HV = a.HV, K = a.K, V = a.V;
  const int nvs = (V + VB - 1) / VB;
  const int slice = blockIdx.x % nvs;
  const int nh = blockIdx.x / nvs, n = nh / HV, hv = nh - n * HV;
  const int hq = hv / (HV / H);
  const int v0 = slice * VB;
  int64_t bos, Tn;
  if (a.cu) {
    bos = a.cu[n];
    Tn = a.cu[n + 1] - bos;
  } else {
    bos = (int64_t)n * a.T;
    Tn = a.T;
  }
  const float* h0p = nullptr;
  float* htp = nullptr;
  if (a.state_idx) {
    const int64_t slot = a.state_idx[n];
    if (slot < 0) return;  // padded slot: nothing to do
    if (a.h0) h0p = a.h0 + slot * a.state_stride + (int64_t)hv * K * V;
    if (a.ht) htp = a.ht + slot * a.state_stride + (int64_t)hv * K * V;
  } else {
    if (a.h0) h0p = a.h0 + ((int64_t)n * HV + hv) * K * V;
    if (a.ht) htp = a.ht + ((int64_t)n * HV + hv) * K * V;
  }

  const int cg = tid % CG, rg = tid / CG;
  const int col0 = 4 * cg;           // within the slice
  const int gcol = v0 + col0;        // within the state row
  const bool vec = (V % 4) == 0;
  float S[RPT][4];
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int r = rg * RPT + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) S[i][j] = 0.f;
    if (h0p && r < K) {
      if (vec && gcol < V) {
        float4 x = __ldcs(reinterpret_cast<const float4*>(h0p + (int64_t)r * V + gcol));
        S[i][0] = x.x; S[i][1] = x.y; S[i][2] = x.z; S[i][3] = x.w;
      } else if (!vec) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (gcol + j < V) S[i][j] = h0p[(int64_t)r * V + gcol + j];
      }
    }
  }

  const T* q = reinterpret_cast<const T*>(a.q);
  const T* k = reinterpret_cast<const T*>(a.k);
  const T* v = reinterpret_cast<const T*>(a.v);
  const T* b = reinterpret_cast<const T*>(a.b);
  const T* w = reinterpret_cast<const T*>(a.w);
  T* o = reinterpret_cast<T*>(a.o);
  for (int64_t t = 0; t < Tn; ++t) {
    const int64_t row = bos + t;
    const int64_t oq = (row * H + hq) * K, og = (row * HV + hv) * K, ov = (row * HV + hv) * V;
    for (int idx = tid; idx < D; idx += blockDim.x) {
      const bool kk = idx < K;
      sq[idx] = kk ? to_f<T>(q[oq + idx]) : 0.f;
      sk[idx] = kk ? to_f<T>(k[oq + idx]) : 0.f;
      sg[idx] = kk ? expf(a.g[og + idx]) : 0.f;
      sb[idx] = kk ? to_f<T>(b[og + idx]) : 0.f;
    }
    for (int idx = tid; idx < VB; idx += blockDim.x) {
      const bool vv = v0 + idx < V;
      sv[idx] = vv ? to_f<T>(v[ov + v0 + idx]) : 0.f;
      sw[idx] = vv ? to_f<T>(w[ov + v0 + idx]) : 0.f;
    }
    __syncthreads();
    if (warp < 2) {
      const float* x = warp == 0 ? sq : sk;
      float s = 0.f;
      for (int idx = lane; idx < D; idx += 32) s += x[idx] * x[idx];
      s = warp_sum(s);
      if (lane == 0) {
        const float inv = a.l2norm ? rsqrtf(s + kNormEps) : 1.f;
        snorm[warp] = warp == 0 ? inv * a.scale : inv;
      }
    }
    __syncthreads();
    const float nq = snorm[0], nk = snorm[1];
    // decay, then erase-read r = S^T (b*k)
    float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg * RPT + i;
      const float dec = sg[r], kb = sb[r] * sk[r] * nk;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S[i][j] *= dec;
        part[j] += S[i][j] * kb;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[rg][col0 + j] = part[j];
    __syncthreads();
    float dlt[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float s = 0.f;
#pragma unroll
      for (int x = 0; x < RG; ++x) s += red[x][col0 + j];
      dlt[j] = sw[col0 + j] * sv[col0 + j] - s;
    }
    __syncthreads();
    // rank-1 write and read-out
#pragma unroll
    for (int j = 0; j < 4; ++j) part[j] = 0.f;
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg * RPT + i;
      const float kr = sk[r] * nk, qr = sq[r] * nq;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        S[i][j] += kr * dlt[j];
        part[j] += S[i][j] * qr;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[rg][col0 + j] = part[j];
    __syncthreads();
    for (int idx = tid; idx < VB; idx += blockDim.x) {
      if (v0 + idx < V) {
        float s = 0.f;
#pragma unroll
        for (int x = 0; x < RG; ++x) s += red[x][idx];
        o[ov + v0 + idx] = from_f<T>(s);
      }
    }
    __syncthreads();
  }

  if (htp) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg * RPT + i;
      if (r < K) {
        if (vec && gcol < V) {
          __stcs(reinterpret_cast<float4*>(htp + (int64_t)r * V + gcol),
                 make_float4(S[i][0], S[i][1], S[i][2], S[i][3]));
        } else if (!vec) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (gcol + j < V) htp[(int64_t)r * V + gcol + j] = S[i][j];
        }
      }
    }
  }
}

template <typename T, int D>
cudaError_t launch_recurrent(const RecArgs& a, cudaStream_t st) {
  constexpr int VB = 64;
  const int nvs = (a.V + VB - 1) / VB;
  dim3 grid(a.n_seqs * a.HV * nvs);
  k_recurrent<T, D, VB><<<grid, kThreads, 0, st>>>(a);
  return cudaGetLastError();
}

#define GDN2_INST_REC(T, D) template cudaError_t launch_recurrent<T, D>(const RecArgs&, cudaStream_t);
GDN2_INST_REC(float, 64)
GDN2_INST_REC(float, 128)
GDN2_INST_REC(__nv_bfloat16, 64)
GDN2_INST_REC(__nv_bfloat16, 128)
GDN2_INST_REC(__half, 64)
GDN2_INST_REC(__half, 128)

}  // namespace gdn2
