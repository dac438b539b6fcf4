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
#include "tc.cuh"

namespace gdn2 {

// Log-decay of channel c from the raw gate input x (gate in kernel,
// fused_recurrent_gdn2.py:257-272); hq is the key head.
__device__ __forceinline__ float gate_logdecay(const RecArgs& a, float x, int hq, int c) {
  if (a.gate == 0) return x;
  if (a.dt_bias) x += a.dt_bias[hq * a.K + c];
  const float A = expf(a.A_log[hq]);
  if (a.gate == 2) return a.lower_bound / (1.f + expf(-A * x));  // lower_bound * sigmoid(A x)
  const float sp = x > 20.f ? x : log1pf(expf(x));               // softplus
  return -A * sp;
}


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
  const int32_t* tok_idx = nullptr;  // speculative decoding: a slot per token
  if (a.state_idx) {
    int64_t slot;
    if (a.idx_stride > 0) {
      tok_idx = a.state_idx + (int64_t)n * a.idx_stride;
      const int acc = a.n_accepted ? a.n_accepted[n] : 1;
      slot = acc >= 1 ? tok_idx[acc - 1] : -1;
    } else {
      slot = a.state_idx[n];
    }
    if (slot < 0) return;  // padded slot: nothing to do
    if (a.h0) h0p = a.h0 + slot * a.state_stride + (int64_t)hv * K * V;
    if (a.ht && !tok_idx) htp = a.ht + slot * a.state_stride + (int64_t)hv * K * V;
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

  auto store_state = [&](float* dst) {
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg * RPT + i;
      if (r < K) {
        if (vec && gcol < V) {
          __stcs(reinterpret_cast<float4*>(dst + (int64_t)r * V + gcol),
                 make_float4(S[i][0], S[i][1], S[i][2], S[i][3]));
        } else if (!vec) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (gcol + j < V) dst[(int64_t)r * V + gcol + j] = S[i][j];
        }
      }
    }
  };

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
      sg[idx] = kk ? expf(gate_logdecay(a, a.g[og + idx], hq, idx)) : 0.f;
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
    if (tok_idx && a.ht) {  // the state after token t goes to its own slot
      const int64_t slot = tok_idx[t];
      if (slot >= 0) store_state(a.ht + slot * a.state_stride + (int64_t)hv * K * V);
    }
  }

  if (htp) store_state(htp);
}

// ---------------------------------------------------------------------------
// Streaming variant for full states (K = V = D): a persistent CTA of 512
// threads per SM walks (sequence, value head) units.  Each unit's whole fp32
// state (D x D, contiguous) and its first token's q, k, b, g, v, w arrive by
// 1-D bulk async copies into a three-buffer shared-memory ring two units ahead,
// so HBM streams the next state while this one is updated; the new state
// leaves from registers with 128-bit streaming stores.  Same arithmetic,
// order and reductions as k_recurrent (thread (rg, cg) holds rows
// [rg*RPT, +RPT) x columns [4cg, 4cg+4)); every warp forms the q / k norms
// itself and the two column reductions have separate buffers, so a token
// costs four block barriers.
struct RecUnit {
  int64_t bos, Tn;
  const float* h0;
  float* ht;
  const int32_t* tok_idx;  // speculative decoding: the state slot of each token
  int hv, hq, skip;
};

__device__ __forceinline__ RecUnit rec_unit(const RecArgs& a, int u) {
  RecUnit r;
  const int n = u / a.HV, hv = u - (u / a.HV) * a.HV;
  r.hv = hv;
  r.hq = hv / (a.HV / a.H);
  if (a.cu) {
    r.bos = a.cu[n];
    r.Tn = a.cu[n + 1] - r.bos;
  } else {
    r.bos = (int64_t)n * a.T;
    r.Tn = a.T;
  }
  r.h0 = nullptr;
  r.ht = nullptr;
  r.tok_idx = nullptr;
  r.skip = 0;
  const int64_t KV = (int64_t)a.K * a.V;
  if (a.state_idx) {
    int64_t slot;
    if (a.idx_stride > 0) {
      r.tok_idx = a.state_idx + (int64_t)n * a.idx_stride;
      const int acc = a.n_accepted ? a.n_accepted[n] : 1;
      slot = acc >= 1 ? r.tok_idx[acc - 1] : -1;
    } else {
      slot = a.state_idx[n];
    }
    if (slot < 0) {
      r.skip = 1;
      return r;
    }
    if (a.h0) r.h0 = a.h0 + slot * a.state_stride + (int64_t)hv * KV;
    if (a.ht && !r.tok_idx) r.ht = a.ht + slot * a.state_stride + (int64_t)hv * KV;
  } else {
    if (a.h0) r.h0 = a.h0 + ((int64_t)n * a.HV + hv) * KV;
    if (a.ht) r.ht = a.ht + ((int64_t)n * a.HV + hv) * KV;
  }
  return r;
}

template <int D>
struct RecStreamSmem {
  static constexpr int NTH = 512;
  static constexpr int NBUF = 3;
  static constexpr int CG = D / 4, RG = NTH / CG, RPT = D / RG;
  static constexpr uint32_t state = D * D * 4;     // one state buffer
  static constexpr uint32_t raw = 24 * D;           // q, k, b, v, w (<= 4 B each) and g of one token
  static constexpr uint32_t oState = 0;
  static constexpr uint32_t oRaw = NBUF * state;
  static constexpr uint32_t oF = oRaw + NBUF * raw;                // sq sk sg sb sv sw floats
  static constexpr uint32_t oRed = oF + 6 * D * 4;                 // red[2][RG][D]
  static constexpr uint32_t oUnit = oRed + 2 * RG * D * 4;         // RecUnit[NBUF]
  static constexpr uint32_t oBar = oUnit + NBUF * sizeof(RecUnit);  // mbarrier[NBUF]
  static constexpr uint32_t bytes = oBar + 8 * NBUF + 128;
};

template <typename T, int D>
__global__ void __launch_bounds__(512, 1) k_recurrent_stream(RecArgs a) {
  using S_ = RecStreamSmem<D>;
  constexpr int NTH = S_::NTH, CG = S_::CG, RG = S_::RG, RPT = S_::RPT, NBUF = S_::NBUF;
  constexpr int EB = (int)sizeof(T);
  extern __shared__ __align__(128) unsigned char sm[];
  float* sq = reinterpret_cast<float*>(sm + S_::oF);
  float* sk = sq + D;
  float* sg = sk + D;
  float* sb = sg + D;
  float* sv = sb + D;
  float* sw = sv + D;
  // column partial sums over the row groups: red0 for the erase-read, red1
  // for the read-out, so one barrier per reduction is enough
  float(*red0)[D] = reinterpret_cast<float(*)[D]>(sm + S_::oRed);
  float(*red1)[D] = red0 + RG;
  RecUnit* sUnit = reinterpret_cast<RecUnit*>(sm + S_::oUnit);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + S_::oBar);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int H = a.H, HV = a.HV;
  const int n_units = a.n_seqs * HV;
  const int cg = tid % CG, rg = tid / CG, col0 = 4 * cg;
  const T* q = reinterpret_cast<const T*>(a.q);
  const T* k = reinterpret_cast<const T*>(a.k);
  const T* v = reinterpret_cast<const T*>(a.v);
  const T* b = reinterpret_cast<const T*>(a.b);
  const T* w = reinterpret_cast<const T*>(a.w);
  T* o = reinterpret_cast<T*>(a.o);

  // raw token buffer: q k b (D*EB each) | g (D*4) | v w (D*EB each)
  auto raw_q = [&](int buf) { return sm + S_::oRaw + buf * S_::raw; };
  auto issue = [&](int u, int buf) {  // thread 0
    const RecUnit ui = rec_unit(a, u);
    sUnit[buf] = ui;
    uint32_t bytes = 0;
    const bool st = !ui.skip && ui.h0;
    const bool tok = !ui.skip && ui.Tn > 0;
    if (st) bytes += S_::state;
    if (tok) bytes += 5 * D * EB + D * 4;
    tc::mbar_expect_tx(&bar[buf], bytes);
    if (st) tc::bulk_load(sm + S_::oState + buf * S_::state, ui.h0, S_::state, &bar[buf]);
    if (tok) {
      const int64_t oq = (ui.bos * H + ui.hq) * D, og = (ui.bos * HV + ui.hv) * D;
      unsigned char* r = raw_q(buf);
      tc::bulk_load(r, q + oq, D * EB, &bar[buf]);
      tc::bulk_load(r + D * EB, k + oq, D * EB, &bar[buf]);
      tc::bulk_load(r + 2 * D * EB, b + og, D * EB, &bar[buf]);
      tc::bulk_load(r + 3 * D * EB, a.g + og, D * 4, &bar[buf]);
      tc::bulk_load(r + 3 * D * EB + D * 4, v + og, D * EB, &bar[buf]);
      tc::bulk_load(r + 4 * D * EB + D * 4, w + og, D * EB, &bar[buf]);
    }
  };

  if (tid == 0) {
    for (int i = 0; i < NBUF; ++i) tc::mbar_init(&bar[i], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int i = 0; i < NBUF - 1; ++i)
      if ((int)blockIdx.x + i * (int)gridDim.x < n_units) issue(blockIdx.x + i * gridDim.x, i);

  int fault = 0;
  int it = 0;  // after a fault: the iteration whose copy did not land
  for (int u = blockIdx.x; u < n_units; u += gridDim.x, ++it) {
    const int buf = it % NBUF;
    const uint32_t par = (uint32_t)(it / NBUF) & 1u;
    if (!tc::mbar_wait(&bar[buf], par)) fault = 1;
    if (__syncthreads_or(fault)) break;
    // the buffer NBUF-1 units ahead held the previous unit, which is done (its
    // state went to registers and its token was read before its last barrier)
    {
      const int ahead = u + (NBUF - 1) * (int)gridDim.x;
      if (tid == 0 && ahead < n_units) issue(ahead, (it + NBUF - 1) % NBUF);
    }
    const RecUnit ui = sUnit[buf];
    if (ui.skip) continue;

    float S[RPT][4];
    const float* st = reinterpret_cast<const float*>(sm + S_::oState + buf * S_::state);
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
      const int r = rg * RPT + i;
      if (ui.h0) {
        const float4 x = *reinterpret_cast<const float4*>(st + r * D + col0);
        S[i][0] = x.x; S[i][1] = x.y; S[i][2] = x.z; S[i][3] = x.w;
      } else {
        S[i][0] = S[i][1] = S[i][2] = S[i][3] = 0.f;
      }
    }

    for (int64_t t = 0; t < ui.Tn; ++t) {
      const int64_t row = ui.bos + t;
      const int64_t oq = (row * H + ui.hq) * D, og = (row * HV + ui.hv) * D;
      if (t > 0) __syncthreads();  // the previous token's read-out is done with sq .. sw, red1
      if (t == 0) {
        const unsigned char* r = raw_q(buf);
        for (int idx = tid; idx < D; idx += NTH) {
          sq[idx] = to_f<T>(reinterpret_cast<const T*>(r)[idx]);
          sk[idx] = to_f<T>(reinterpret_cast<const T*>(r + D * EB)[idx]);
          sb[idx] = to_f<T>(reinterpret_cast<const T*>(r + 2 * D * EB)[idx]);
          sg[idx] = expf(gate_logdecay(a, reinterpret_cast<const float*>(r + 3 * D * EB)[idx],
                                       ui.hq, idx));
          sv[idx] = to_f<T>(reinterpret_cast<const T*>(r + 3 * D * EB + D * 4)[idx]);
          sw[idx] = to_f<T>(reinterpret_cast<const T*>(r + 4 * D * EB + D * 4)[idx]);
        }
      } else {
        for (int idx = tid; idx < D; idx += NTH) {
          sq[idx] = to_f<T>(q[oq + idx]);
          sk[idx] = to_f<T>(k[oq + idx]);
          sb[idx] = to_f<T>(b[og + idx]);
          sg[idx] = expf(gate_logdecay(a, a.g[og + idx], ui.hq, idx));
          sv[idx] = to_f<T>(v[og + idx]);
          sw[idx] = to_f<T>(w[og + idx]);
        }
      }
      __syncthreads();
      // every warp forms the q and k norms itself (no barrier)
      float nq, nk;
      {
        float s1 = 0.f, s2 = 0.f;
        for (int idx = lane; idx < D; idx += 32) {
          s1 += sq[idx] * sq[idx];
          s2 += sk[idx] * sk[idx];
        }
        s1 = warp_sum(s1);
        s2 = warp_sum(s2);
        nq = (a.l2norm ? rsqrtf(s1 + kNormEps) : 1.f) * a.scale;
        nk = a.l2norm ? rsqrtf(s2 + kNormEps) : 1.f;
      }
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
      for (int j = 0; j < 4; ++j) red0[rg][col0 + j] = part[j];
      __syncthreads();
      float dlt[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float s = 0.f;
#pragma unroll
        for (int x = 0; x < RG; ++x) s += red0[x][col0 + j];
        dlt[j] = sw[col0 + j] * sv[col0 + j] - s;
      }
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
      for (int j = 0; j < 4; ++j) red1[rg][col0 + j] = part[j];
      __syncthreads();
      for (int idx = tid; idx < D; idx += NTH) {
        float s = 0.f;
#pragma unroll
        for (int x = 0; x < RG; ++x) s += red1[x][idx];
        o[og + idx] = from_f<T>(s);
      }
      // (the next token's first barrier, or the next unit's, orders these
      // reads of red1 and sq .. sw before they are overwritten)
      if (ui.tok_idx && a.ht) {  // the state after token t goes to its own slot
        const int64_t slot = ui.tok_idx[t];
        if (slot >= 0) {
          float* dst = a.ht + slot * a.state_stride + (int64_t)ui.hv * D * D;
#pragma unroll
          for (int i = 0; i < RPT; ++i)
            __stcs(reinterpret_cast<float4*>(dst + (int64_t)(rg * RPT + i) * D + col0),
                   make_float4(S[i][0], S[i][1], S[i][2], S[i][3]));
        }
      }
    }

    if (ui.ht) {
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const int r = rg * RPT + i;
        __stcs(reinterpret_cast<float4*>(ui.ht + (int64_t)r * D + col0),
               make_float4(S[i][0], S[i][1], S[i][2], S[i][3]));
      }
    }
  }
  if (fault && tid == 0) {
    // bounded waits: let the copies still in flight land
    for (int j = it; j < it + NBUF - 1; ++j) tc::mbar_wait(&bar[j % NBUF], (uint32_t)(j / NBUF) & 1u);
    atomicOr(a.fault, 4u);
  }
}

// The streaming kernel serves full K = V = D states whose rows and vectors
// are 16-byte aligned (bulk copies); anything else takes k_recurrent.
template <typename T, int D>
bool recurrent_stream_ok(const RecArgs& a) {
  if (a.K != D || a.V != D || !a.fault) return false;
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.q) | reinterpret_cast<uintptr_t>(a.k) |
                       reinterpret_cast<uintptr_t>(a.v) | reinterpret_cast<uintptr_t>(a.b) |
                       reinterpret_cast<uintptr_t>(a.w) | reinterpret_cast<uintptr_t>(a.g) |
                       reinterpret_cast<uintptr_t>(a.h0) | reinterpret_cast<uintptr_t>(a.ht) |
                       reinterpret_cast<uintptr_t>(a.o);
  if ((al & 15) != 0) return false;
  if (a.state_idx && (a.state_stride % 4) != 0) return false;
  return true;
}

template <typename T, int D>
cudaError_t launch_recurrent(const RecArgs& a, cudaStream_t st) {
  if constexpr (D <= 128) {  // a 256 x 256 state ring would not fit shared memory
   if (recurrent_stream_ok<T, D>(a)) {
    const int n_units = a.n_seqs * a.HV;
    if (n_units == 0) return cudaSuccess;
    auto kern = k_recurrent_stream<T, D>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)RecStreamSmem<D>::bytes);
    if (e != cudaSuccess) return e;
    int sms = 0;
    e = num_sms(&sms);
    if (e != cudaSuccess) return e;
    const int grid = n_units < sms ? n_units : sms;
    kern<<<grid, 512, RecStreamSmem<D>::bytes, st>>>(a);
    return cudaGetLastError();
   }
  }
  // 256-row states take 32-column slices (32 state floats per thread, as
  // the 64-column slices of 128-row states)
  constexpr int VB = D > 128 ? 32 : 64;
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
GDN2_INST_REC(float, 256)
GDN2_INST_REC(__nv_bfloat16, 256)
GDN2_INST_REC(__half, 256)

}  // namespace gdn2
