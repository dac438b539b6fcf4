// abi.cu -- extern "C" entry points of libgdn2_b200.so (declared in
// include/gdn2_b200.h): argument validation, dtype / head-size dispatch,
// per-thread error messages, and the small context-parallel merge kernel.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <string>

#include "../../include/gdn2_b200.h"

#include "chunk_args.cuh"
#include "mma16.cuh"

namespace gdn2 {
template <typename T, int D> cudaError_t launch_fwd_intra(const FwdIntraArgs&, cudaStream_t);
template <typename T, int D> cudaError_t launch_fwd_state(const FwdStateArgs&, cudaStream_t);
template <typename T, int D> cudaError_t launch_bwd_state(const BwdStateArgs&, cudaStream_t);
template <typename T, int D> cudaError_t launch_bwd_intra(const BwdIntraArgs&, cudaStream_t);
template <typename T, int D> cudaError_t launch_recurrent(const RecArgs&, cudaStream_t);
template <typename T, int D, int BV> cudaError_t launch_fwd_state16(const FwdStateArgs&, cudaStream_t);
template <typename T, int D, int BV> cudaError_t launch_bwd_state16(const BwdStateArgs&, cudaStream_t);
template <typename T, int D> cudaError_t launch_bwd_intra16(const BwdIntraArgs&, cudaStream_t);
template <typename T, int D> cudaError_t launch_fwd_intra16(const FwdIntraArgs&, cudaStream_t);
template <typename T> cudaError_t launch_fwd_intra_wide(const FwdIntraArgs&, cudaStream_t);
template <typename T> cudaError_t launch_fwd_state_wide(const FwdStateArgs&, cudaStream_t);
template <typename T> cudaError_t launch_bwd_state_wide(const BwdStateArgs&, cudaStream_t);
template <typename T> cudaError_t launch_bwd_intra_wide(const BwdIntraArgs&, cudaStream_t);
bool fwd_state_tc_ok(const FwdStateArgs&, int dtype_bf16);
cudaError_t launch_fwd_state_tc(const FwdStateArgs&, cudaStream_t);
bool bwd_state_tc_ok(const BwdStateArgs&, int dtype_bf16);
cudaError_t launch_bwd_state_tc(const BwdStateArgs&, cudaStream_t);
cudaError_t read_fault_bits(unsigned int* bits, bool clear);
cudaError_t fault_word(unsigned int** ptr);
}  // namespace gdn2

using namespace gdn2;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* where) {
  return fail(GDN2_ERR_CUDA, "%s: CUDA error %d (%s)", where, (int)e, cudaGetErrorString(e));
}

int esize_of(int dtype) { return dtype == GDN2_DTYPE_F32 ? 4 : 2; }

bool dtype_ok(int dtype) {
  return dtype == GDN2_DTYPE_F32 || dtype == GDN2_DTYPE_BF16 || dtype == GDN2_DTYPE_F16;
}

// Head size bucket: the chunk kernels are compiled for padded head sizes 64
// and 128 (larger heads take chunk_wide.cu), the decode kernel also for 256.
int head_bucket(int K, int V) {
  int m = K > V ? K : V;
  return m <= 64 ? 64 : (m <= 128 ? 128 : 256);
}

int check_problem(const gdn2_chunk_problem* p, const char* fn) {
  if (!p) return fail(GDN2_ERR_INVALID, "%s: null problem", fn);
  if (p->H <= 0 || p->K <= 0 || p->V <= 0)
    return fail(GDN2_ERR_INVALID, "%s: H, K, V must be positive (got %d, %d, %d)", fn, p->H, p->K,
                p->V);
  if (p->K > 256 || p->V > 256)
    return fail(GDN2_ERR_UNSUPPORTED, "%s: head sizes up to 256 are supported (K=%d, V=%d)", fn,
                p->K, p->V);
  if (!dtype_ok(p->dtype)) return fail(GDN2_ERR_INVALID, "%s: unknown dtype %d", fn, p->dtype);
  if (p->seqs.n_seqs < 0 || p->seqs.n_chunks < 0)
    return fail(GDN2_ERR_INVALID, "%s: negative sequence or chunk count", fn);
  if (p->seqs.n_seqs > 0 && (!p->seqs.cu_seqlens || !p->seqs.chunk_offsets))
    return fail(GDN2_ERR_INVALID, "%s: missing sequence tables", fn);
  if (p->seqs.n_chunks > 0 && !p->seqs.chunk_seq)
    return fail(GDN2_ERR_INVALID, "%s: missing chunk table", fn);
  if ((int64_t)p->seqs.n_chunks * p->H > 2147483647LL)
    return fail(GDN2_ERR_UNSUPPORTED, "%s: too many chunks", fn);
  if (p->max_ctas < 0)
    return fail(GDN2_ERR_INVALID, "%s: max_ctas must be >= 0 (got %d)", fn, p->max_ctas);
  if (p->gate < 0 || p->gate > 2 || (p->gate && !p->A_log))
    return fail(GDN2_ERR_INVALID, "%s: gate %d needs A_log (modes 0..2)", fn, p->gate);
  if (p->gate && !(p->dtype == GDN2_DTYPE_BF16 && p->K % 8 == 0 && p->V % 8 == 0 &&
                   p->K <= 128 && p->V <= 128))
    return fail(GDN2_ERR_UNSUPPORTED,
                "%s: the gate in kernel is served by the bf16 kernels (K, V multiples of 8, "
                "up to 128)", fn);
  return GDN2_OK;
}

GateArgs gate_of(const gdn2_chunk_problem* p) {
  GateArgs g;
  g.A_log = p->A_log;
  g.dt_bias = p->dt_bias;
  g.mode = p->gate;
  g.lower_bound = p->lower_bound;
  g.dA_log = p->dA_log;
  g.ddt_bias = p->ddt_bias;
  return g;
}

Seqs make_seqs(const gdn2_chunk_problem* p) {
  Seqs s;
  s.cu = p->seqs.cu_seqlens;
  s.coff = p->seqs.chunk_offsets;
  s.cseq = p->seqs.chunk_seq;
  s.n_seqs = p->seqs.n_seqs;
  s.n_chunks = p->seqs.n_chunks;
  return s;
}

SavedLayout layout_of(const gdn2_chunk_problem* p) {
  return saved_layout(p->seqs.n_chunks, p->H, p->K, p->V, esize_of(p->dtype));
}

BwdLayout bwd_layout_of(const gdn2_chunk_problem* p) {
  return bwd_layout(p->seqs.n_chunks, p->H, p->K, p->V, esize_of(p->dtype));
}

template <template <typename, int> class F, typename Args>
cudaError_t dispatch(int dtype, int bucket, const Args& a, cudaStream_t st) {
  if (dtype == GDN2_DTYPE_F32)
    return bucket == 64 ? F<float, 64>::run(a, st) : F<float, 128>::run(a, st);
  if (dtype == GDN2_DTYPE_BF16)
    return bucket == 64 ? F<__nv_bfloat16, 64>::run(a, st) : F<__nv_bfloat16, 128>::run(a, st);
  return bucket == 64 ? F<__half, 64>::run(a, st) : F<__half, 128>::run(a, st);
}

template <typename T, int D> struct RunFwdIntra {
  static cudaError_t run(const FwdIntraArgs& a, cudaStream_t s) { return launch_fwd_intra<T, D>(a, s); }
};
template <typename T, int D> struct RunFwdState {
  static cudaError_t run(const FwdStateArgs& a, cudaStream_t s) { return launch_fwd_state<T, D>(a, s); }
};
template <typename T, int D> struct RunBwdState {
  static cudaError_t run(const BwdStateArgs& a, cudaStream_t s) { return launch_bwd_state<T, D>(a, s); }
};
template <typename T, int D> struct RunBwdIntra {
  static cudaError_t run(const BwdIntraArgs& a, cudaStream_t s) { return launch_bwd_intra<T, D>(a, s); }
};
template <typename T, int D> struct RunRec {
  static cudaError_t run(const RecArgs& a, cudaStream_t s) { return launch_recurrent<T, D>(a, s); }
};
cudaError_t dispatch_rec(int dtype, int bucket, const RecArgs& a, cudaStream_t st) {
  if (bucket == 256) {
    if (dtype == GDN2_DTYPE_F32) return launch_recurrent<float, 256>(a, st);
    if (dtype == GDN2_DTYPE_BF16) return launch_recurrent<__nv_bfloat16, 256>(a, st);
    return launch_recurrent<__half, 256>(a, st);
  }
  return dispatch<RunRec>(dtype, bucket, a, st);
}

// State passes: 16-bit inputs whose head sizes are multiples of 8 take the
// ldmatrix / m16n8k16 kernels (state16.cu); everything else the generic ones.
// The value tile is 128 columns when that still gives one CTA per SM or more,
// else 64.
template <typename T, int D, int BV>
cudaError_t launch_state16(const FwdStateArgs& a, cudaStream_t st) {
  return launch_fwd_state16<T, D, BV>(a, st);
}
template <typename T, int D, int BV>
cudaError_t launch_state16(const BwdStateArgs& a, cudaStream_t st) {
  return launch_bwd_state16<T, D, BV>(a, st);
}

// Column slices of 64 double the CTAs of a latency-bound pass; only worth it
// while the doubled grid still fits one wave (a CTA walks all of its
// sequence's chunks, so a second wave would start only after the first ends).
template <typename T, typename Args>
cudaError_t run_state16(const Args& a, int bucket, int cols, int n_seqs, int H, cudaStream_t st) {
  if (bucket == 64) return launch_state16<T, 64, 64>(a, st);
  const long ctas128 = (long)n_seqs * H * ((cols + 127) / 128);
  if (2 * ctas128 > 148) return launch_state16<T, 128, 128>(a, st);
  return launch_state16<T, 128, 64>(a, st);
}

// The ldmatrix / m16n8k16 kernels serve bf16 with head sizes that are
// multiples of 8.  Their decay-scaled operands span up to 2^+-100, which
// bf16 represents (8-bit exponent) and fp16 does not, so fp16 problems stay
// on the fp32-staged kernels.
bool use16(const gdn2_chunk_problem* p) {
  return p->dtype == GDN2_DTYPE_BF16 && (p->K % 8) == 0 && (p->V % 8) == 0 && p->K <= 128 &&
         p->V <= 128;
}

// Heads above 128 channels (K or V) take the slab-walking kernels of
// chunk_wide.cu, for every dtype.
bool use_wide(const gdn2_chunk_problem* p) { return wide_heads(p->K, p->V); }

template <template <typename> class F, typename Args>
cudaError_t dispatch_wide(int dtype, const Args& a, cudaStream_t st) {
  if (dtype == GDN2_DTYPE_F32) return F<float>::run(a, st);
  if (dtype == GDN2_DTYPE_BF16) return F<__nv_bfloat16>::run(a, st);
  return F<__half>::run(a, st);
}
template <typename T> struct RunFwdIntraW {
  static cudaError_t run(const FwdIntraArgs& a, cudaStream_t s) { return launch_fwd_intra_wide<T>(a, s); }
};
template <typename T> struct RunFwdStateW {
  static cudaError_t run(const FwdStateArgs& a, cudaStream_t s) { return launch_fwd_state_wide<T>(a, s); }
};
template <typename T> struct RunBwdStateW {
  static cudaError_t run(const BwdStateArgs& a, cudaStream_t s) { return launch_bwd_state_wide<T>(a, s); }
};
template <typename T> struct RunBwdIntraW {
  static cudaError_t run(const BwdIntraArgs& a, cudaStream_t s) { return launch_bwd_intra_wide<T>(a, s); }
};

bool aligned16(const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; }

// The 16-bit kernels move token rows with bulk async copies, which need
// 16-byte aligned rows.
int check_aligned16(const gdn2_chunk_problem* p, const char* fn,
                    std::initializer_list<const void*> ptrs) {
  if (!use16(p)) return GDN2_OK;
  for (const void* x : ptrs)
    if (x && !aligned16(x))
      return fail(GDN2_ERR_INVALID,
                  "%s: bf16 tensors must start on a 16-byte boundary (got %p)", fn, x);
  return GDN2_OK;
}

// bf16 with K = V = 128 (the pre-scan excepted) runs the forward state pass
// on tcgen05 / TMEM / TMA (state_tc.cu).
cudaError_t fwd_state_dispatch(const gdn2_chunk_problem* p, const FwdStateArgs& a, cudaStream_t st) {
  if (use_wide(p)) return dispatch_wide<RunFwdStateW>(p->dtype, a, st);
  const int bucket = head_bucket(p->K, p->V);
  if (fwd_state_tc_ok(a, p->dtype == GDN2_DTYPE_BF16)) return launch_fwd_state_tc(a, st);
  if (use16(p)) {
    const int cols = a.prescan ? p->V + p->K : p->V;
    return run_state16<__nv_bfloat16>(a, bucket, cols, p->seqs.n_seqs, p->H, st);
  }
  return dispatch<RunFwdState>(p->dtype, bucket, a, st);
}

cudaError_t bwd_state_dispatch(const gdn2_chunk_problem* p, const BwdStateArgs& a, cudaStream_t st) {
  if (use_wide(p)) return dispatch_wide<RunBwdStateW>(p->dtype, a, st);
  const int bucket = head_bucket(p->K, p->V);
  if (bwd_state_tc_ok(a, p->dtype == GDN2_DTYPE_BF16)) return launch_bwd_state_tc(a, st);
  if (use16(p)) {
    return run_state16<__nv_bfloat16>(a, bucket, p->V, p->seqs.n_seqs, p->H, st);
  }
  return dispatch<RunBwdState>(p->dtype, bucket, a, st);
}

cudaError_t fwd_intra_dispatch(const gdn2_chunk_problem* p, const FwdIntraArgs& a, cudaStream_t st) {
  if (use_wide(p)) return dispatch_wide<RunFwdIntraW>(p->dtype, a, st);
  const int bucket = head_bucket(p->K, p->V);
  if (use16(p)) {
    return bucket == 64 ? launch_fwd_intra16<__nv_bfloat16, 64>(a, st)
                        : launch_fwd_intra16<__nv_bfloat16, 128>(a, st);
  }
  return dispatch<RunFwdIntra>(p->dtype, bucket, a, st);
}

cudaError_t bwd_intra_dispatch(const gdn2_chunk_problem* p, const BwdIntraArgs& a, cudaStream_t st) {
  if (use_wide(p)) return dispatch_wide<RunBwdIntraW>(p->dtype, a, st);
  const int bucket = head_bucket(p->K, p->V);
  if (use16(p)) {
    return bucket == 64 ? launch_bwd_intra16<__nv_bfloat16, 64>(a, st)
                        : launch_bwd_intra16<__nv_bfloat16, 128>(a, st);
  }
  return dispatch<RunBwdIntra>(p->dtype, bucket, a, st);
}

// ---- context-parallel merge ----------------------------------------------
// One CTA per (sequence, head, 32-column tile of the state).  The running
// tile x (K x 32, fp32) and its successor stay in shared memory; for each
// folded rank j the CTA applies x <- M_j x + h_e_j (forward) or
// x <- M_j^T x + dh_j (backward), staging M_j in blocks of 64 output rows
// (64 x K rows of M, or K x 64 columns of it for the transpose, read
// coalesced) and multiplying on the tensor cores with the 3-term TF32 split
// (about fp32 accuracy).
constexpr int kMergeRows = 64;
constexpr int kMergeLDX = 32 + 4;
constexpr int kMergeLDB = kMergeRows + 4;  // row stride of a staged K x 64 column block

__host__ __device__ inline int merge_depth(int K) { return (K + 7) & ~7; }
// floats of the staged block: 64 rows of M (stride depth + 4) or depth rows
// of 64 columns (stride kMergeLDB)
__host__ __device__ inline int merge_block_floats(int K) {
  const int kd = merge_depth(K);
  const int f = kMergeRows * (kd + 4), b = kd * kMergeLDB;
  return f > b ? f : b;
}
size_t merge_smem_bytes(int K) {
  return (size_t)(2 * merge_depth(K) * kMergeLDX + merge_block_floats(K)) * sizeof(float);
}

__global__ void __launch_bounds__(kThreads) k_cp_merge(int N, int H, int K, int V,
                                                      const float* hm_all, const float* dhm_all,
                                                      int rank, int world, int forward,
                                                      const float* init, float* out) {
  extern __shared__ __align__(16) float smem[];
  const int kd = merge_depth(K);  // product depth; rows K .. kd-1 of x stay zero
  const int ldm = forward ? kd + 4 : kMergeLDB;
  float* x = smem;
  float* y = x + kd * kMergeLDX;
  float* sM = y + kd * kMergeLDX;
  const int nh = blockIdx.y, v0 = blockIdx.x * 32;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int VK = V + K;
  const int64_t per_rank_hm = (int64_t)N * H * K * VK;
  const int64_t per_rank_dh = (int64_t)N * H * K * V;
  for (int idx = tid; idx < kd * 32; idx += kThreads) {
    const int r = idx >> 5, c = idx & 31, col = v0 + c;
    x[r * kMergeLDX + c] =
        (init && r < K && col < V) ? init[((int64_t)nh * K + r) * V + col] : 0.f;
    y[r * kMergeLDX + c] = 0.f;
  }
  __syncthreads();
  const int m0 = (warp & 3) * 16, n0 = (warp >> 2) * 16;
  for (int step = 0; step < (forward ? rank : world - 1 - rank); ++step) {
    const int j = forward ? step : world - 1 - step;
    const float* hm = hm_all + j * per_rank_hm + (int64_t)nh * K * VK;
    for (int r0 = 0; r0 < K; r0 += kMergeRows) {
      const int nr = min(kMergeRows, K - r0);
      // stage the block of M (rows r0.. of M, or its columns r0.. for M^T)
      if (forward) {
        for (int idx = tid; idx < kMergeRows * kd; idx += kThreads) {
          const int r = idx / kd, m = idx - r * kd;
          sM[r * ldm + m] = (r < nr && m < K) ? hm[(int64_t)(r0 + r) * VK + V + m] : 0.f;
        }
      } else {
        for (int idx = tid; idx < kd * kMergeRows; idx += kThreads) {
          const int m = idx / kMergeRows, r = idx - m * kMergeRows;
          sM[m * ldm + r] = (r < nr && m < K) ? hm[(int64_t)m * VK + V + r0 + r] : 0.f;
        }
      }
      __syncthreads();
      float acc[1][2][4];
      acc_zero(acc);
      if (forward)
        warp_mma<1, 2, 3>(acc, sM + m0 * ldm, ldm, 1, x + n0, kMergeLDX, 1, kd);
      else
        warp_mma<1, 2, 3>(acc, sM + m0, 1, ldm, x + n0, kMergeLDX, 1, kd);
      acc_foreach(acc, [&](int rr, int cc, float val) {
        const int r = r0 + m0 + rr, c = n0 + cc, col = v0 + c;
        if (r < K) {
          float b = 0.f;
          if (col < V)
            b = forward ? hm[(int64_t)r * VK + col]
                        : dhm_all[j * per_rank_dh + ((int64_t)nh * K + r) * V + col];
          y[r * kMergeLDX + c] = val + b;
        }
      });
      __syncthreads();
    }
    float* t = x;
    x = y;
    y = t;
  }
  for (int idx = tid; idx < K * 32; idx += kThreads) {
    const int r = idx >> 5, c = idx & 31, col = v0 + c;
    if (col < V) out[((int64_t)nh * K + r) * V + col] = x[r * kMergeLDX + c];
  }
}

// The same fold for K <= 128 (a multiple of 16, V a multiple of 4): the whole
// M of the next folded rank and its state slice arrive by 16-byte cp.async
// while the current fold multiplies, so each fold costs its products and not
// a round trip to memory.  M stays row-major in both directions (the
// backward reads it transposed); the row strides keep both fragment reads
// free of bank conflicts.
constexpr int kMerge2MaxK = 128;
size_t merge2_smem_bytes() {
  return (size_t)(4 * kMerge2MaxK * kMergeLDX + 2 * kMerge2MaxK * 136) * sizeof(float);
}

// With `all` set the kernel also writes every intermediate tile: all[0] is
// the initial tile and all[s + 1] the tile after fold s (forward), or
// all[world - 1] the initial tile and all[world - 2 - s] the tile after fold s
// (backward) -- the start states (end-state gradients) of consecutive
// sub-spans.  `out` may then be null.
__global__ void __launch_bounds__(kThreads) k_cp_merge2(int N, int H, int K, int V,
                                                       const float* hm_all, const float* dhm_all,
                                                       int rank, int world, int forward,
                                                       const float* init, float* out,
                                                       float* all) {
  extern __shared__ __align__(16) float smem[];
  const int ldm = forward ? 132 : 136;
  float* x = smem;                                // [128][36] running tile
  float* y = x + kMerge2MaxK * kMergeLDX;         // its successor
  float* hb = y + kMerge2MaxK * kMergeLDX;        // [2][128][36] h_e_j / dh_j slices
  float* Mb = hb + 2 * kMerge2MaxK * kMergeLDX;   // [2][128][136] M_j
  const int nh = blockIdx.y, v0 = blockIdx.x * 32;
  const int tid = threadIdx.x, warp = tid >> 5;
  const int VK = V + K;
  const int64_t per_rank_hm = (int64_t)N * H * K * VK;
  const int64_t per_rank_dh = (int64_t)N * H * K * V;
  const int nsteps = forward ? rank : world - 1 - rank;
  auto issue = [&](int step, int buf) {
    const int j = forward ? step : world - 1 - step;
    const float* hm = hm_all + j * per_rank_hm + (int64_t)nh * K * VK;
    float* sM = Mb + buf * kMerge2MaxK * 136;
    const int cpr = K / 4;  // 16-byte chunks per row of M
    for (int idx = tid; idx < K * cpr; idx += kThreads) {
      const int r = idx / cpr, c4 = idx - r * cpr;
      cp_async16(sM + r * ldm + 4 * c4, hm + (int64_t)r * VK + V + 4 * c4, true);
    }
    float* sh = hb + buf * kMerge2MaxK * kMergeLDX;
    for (int idx = tid; idx < K * 8; idx += kThreads) {
      const int r = idx >> 3, col = v0 + 4 * (idx & 7);
      const float* src = forward ? hm + (int64_t)r * VK + col
                                 : dhm_all + j * per_rank_dh + ((int64_t)nh * K + r) * V + col;
      cp_async16(sh + r * kMergeLDX + 4 * (idx & 7), col < V ? src : hm, col < V);
    }
    cp_async_commit();
  };
  // one intermediate tile of `all` (index i) from the running tile
  auto write_all = [&](const float* t, int i) {
    for (int idx = tid; idx < K * 32; idx += kThreads) {
      const int r = idx >> 5, c = idx & 31, col = v0 + c;
      if (col < V) all[i * per_rank_dh + ((int64_t)nh * K + r) * V + col] = t[r * kMergeLDX + c];
    }
  };
  for (int idx = tid; idx < K * 32; idx += kThreads) {
    const int r = idx >> 5, c = idx & 31, col = v0 + c;
    x[r * kMergeLDX + c] = (init && col < V) ? init[((int64_t)nh * K + r) * V + col] : 0.f;
  }
  if (all) write_all(x, forward ? 0 : world - 1);  // (each thread its own elements)
  if (nsteps > 0) issue(0, 0);
  for (int step = 0; step < nsteps; ++step) {
    const int buf = step & 1;
    if (step + 1 < nsteps) {
      issue(step + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();  // M_j, its slice and the running tile are in
    const float* sM = Mb + buf * kMerge2MaxK * 136;
    const float* sh = hb + buf * kMerge2MaxK * kMergeLDX;
    if (16 * warp < K) {  // warp w: output rows 16 w .. 16 w + 15, all 32 columns
      float acc[1][4][4];
      acc_zero(acc);
      if (forward)
        warp_mma<1, 4, 3>(acc, sM + 16 * warp * ldm, ldm, 1, x, kMergeLDX, 1, K);
      else
        warp_mma<1, 4, 3>(acc, sM + 16 * warp, 1, ldm, x, kMergeLDX, 1, K);
      acc_foreach(acc, [&](int rr, int cc, float val) {
        const int r = 16 * warp + rr;
        y[r * kMergeLDX + cc] = val + sh[r * kMergeLDX + cc];
      });
    }
    __syncthreads();  // y complete; this step's buffers may be refilled
    if (all) write_all(y, forward ? step + 1 : world - 2 - step);
    float* t = x;
    x = y;
    y = t;
  }
  if (out)
    for (int idx = tid; idx < K * 32; idx += kThreads) {
      const int r = idx >> 5, c = idx & 31, col = v0 + c;
      if (col < V) out[((int64_t)nh * K + r) * V + col] = x[r * kMergeLDX + c];
    }
}

}  // namespace

namespace gdn2 {
// Record an error for gdn2_last_error() from another translation unit of the
// library; returns `code`.
int set_error(int code, const char* msg) {
  g_last_error = msg;
  return code;
}
}  // namespace gdn2

extern "C" {

const char* gdn2_version(void) { return "gdn2_b200 0.1.0 (sm_100a)"; }

const char* gdn2_status_string(int status) {
  switch (status) {
    case GDN2_OK: return "ok";
    case GDN2_ERR_INVALID: return "invalid argument";
    case GDN2_ERR_UNSUPPORTED: return "unsupported configuration";
    case GDN2_ERR_CUDA: return "CUDA error";
    case GDN2_ERR_WORKSPACE: return "buffer too small";
    default: return "unknown status";
  }
}

const char* gdn2_last_error(void) { return g_last_error.c_str(); }

size_t gdn2_chunk_saved_bytes(const gdn2_chunk_problem* p) {
  if (check_problem(p, "gdn2_chunk_saved_bytes") != GDN2_OK) return 0;
  return layout_of(p).total;
}

size_t gdn2_chunk_bwd_workspace_bytes(const gdn2_chunk_problem* p) {
  if (check_problem(p, "gdn2_chunk_bwd_workspace_bytes") != GDN2_OK) return 0;
  return bwd_layout_of(p).total;
}

// The backward pre-scan can run as the tensor-core state pass (bf16, K = V =
// 128), which writes its per-chunk gradient tiles to a backward workspace.
size_t gdn2_cp_workspace_bytes(const gdn2_chunk_problem* p) {
  if (check_problem(p, "gdn2_cp_workspace_bytes") != GDN2_OK) return 0;
  if (p->dtype != GDN2_DTYPE_BF16 || p->K != 128 || p->V != 128) return 0;
  return bwd_layout_of(p).total;
}

int gdn2_chunk_fwd_intra(const gdn2_chunk_problem* p, const void* q, const void* k, const void* v,
                         const float* g, const void* b, const void* w, void* saved,
                         size_t saved_bytes, void* stream) {
  int rc = check_problem(p, "gdn2_chunk_fwd_intra");
  if (rc) return rc;
  if (p->seqs.n_chunks == 0) return GDN2_OK;
  if (!q || !k || !v || !g || !b || !w || !saved)
    return fail(GDN2_ERR_INVALID, "gdn2_chunk_fwd_intra: null tensor pointer");
  SavedLayout L = layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_chunk_fwd_intra: saved buffer %zu < %zu bytes",
                saved_bytes, L.total);
  rc = check_aligned16(p, "gdn2_chunk_fwd_intra", {q, k, v, g, b, w, saved});
  if (rc) return rc;
  FwdIntraArgs a;
  a.seqs = make_seqs(p);
  a.H = p->H; a.K = p->K; a.V = p->V;
  a.scale = p->scale;
  a.l2norm = p->use_qk_l2norm;
  a.gate = gate_of(p);
  a.q = q; a.k = k; a.v = v; a.g = g; a.b = b; a.w = w;
  a.saved = static_cast<unsigned char*>(saved);
  a.L = L;
  a.total_rows = p->seqs.total_tokens;
  a.max_ctas = p->max_ctas;
  cudaError_t e = fault_word(&a.fault);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_chunk_fwd_intra");
  e = fwd_intra_dispatch(p, a, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_chunk_fwd_intra");
}

int gdn2_chunk_fwd_state(const gdn2_chunk_problem* p, const float* h0, void* o, float* ht,
                         void* saved, size_t saved_bytes, void* stream) {
  int rc = check_problem(p, "gdn2_chunk_fwd_state");
  if (rc) return rc;
  if (p->seqs.n_seqs == 0) return GDN2_OK;
  if (!o || !saved) return fail(GDN2_ERR_INVALID, "gdn2_chunk_fwd_state: null o or saved");
  SavedLayout L = layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_chunk_fwd_state: saved buffer %zu < %zu bytes",
                saved_bytes, L.total);
  rc = check_aligned16(p, "gdn2_chunk_fwd_state", {h0, o, ht, saved});
  if (rc) return rc;
  FwdStateArgs a;
  a.seqs = make_seqs(p);
  a.H = p->H; a.K = p->K; a.V = p->V;
  a.h0 = h0; a.o = o; a.ht = ht;
  a.saved = static_cast<unsigned char*>(saved);
  a.L = L;
  a.prescan = 0;
  a.hm = nullptr;
  a.max_ctas = p->max_ctas;
  cudaError_t e = fwd_state_dispatch(p, a, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_chunk_fwd_state");
}

int gdn2_chunk_fwd(const gdn2_chunk_problem* p, const void* q, const void* k, const void* v,
                   const float* g, const void* b, const void* w, const float* h0, void* o,
                   float* ht, void* saved, size_t saved_bytes, void* stream) {
  int rc = gdn2_chunk_fwd_intra(p, q, k, v, g, b, w, saved, saved_bytes, stream);
  if (rc) return rc;
  return gdn2_chunk_fwd_state(p, h0, o, ht, saved, saved_bytes, stream);
}

int gdn2_chunk_bwd_state(const gdn2_chunk_problem* p, const void* saved, size_t saved_bytes,
                         const void* dout, const float* dht, float* dh0, void* workspace,
                         size_t workspace_bytes, void* stream) {
  int rc = check_problem(p, "gdn2_chunk_bwd_state");
  if (rc) return rc;
  if (!saved || !dout) return fail(GDN2_ERR_INVALID, "gdn2_chunk_bwd_state: null tensor pointer");
  SavedLayout L = layout_of(p);
  BwdLayout BL = bwd_layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_chunk_bwd_state: saved buffer %zu < %zu bytes",
                saved_bytes, L.total);
  if (workspace_bytes < BL.total || (!workspace && BL.total))
    return fail(GDN2_ERR_WORKSPACE, "gdn2_chunk_bwd_state: workspace %zu < %zu bytes",
                workspace_bytes, BL.total);
  if (p->seqs.n_seqs == 0) return GDN2_OK;
  rc = check_aligned16(p, "gdn2_chunk_bwd_state", {saved, dout, dht, dh0, workspace});
  if (rc) return rc;
  BwdStateArgs s;
  s.seqs = make_seqs(p);
  s.H = p->H; s.K = p->K; s.V = p->V;
  s.dout = dout; s.dht = dht; s.dh0 = dh0;
  s.saved = static_cast<const unsigned char*>(saved);
  s.L = L;
  s.ws = static_cast<unsigned char*>(workspace);
  s.BL = BL;
  s.prescan = 0;
  s.total_rows = p->seqs.total_tokens;
  s.max_ctas = p->max_ctas;
  cudaError_t e = bwd_state_dispatch(p, s, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_chunk_bwd_state");
}

int gdn2_chunk_bwd_intra(const gdn2_chunk_problem* p, const void* q, const void* k,
                         const void* v, const float* g, const void* b, const void* w,
                         const void* saved, size_t saved_bytes, const void* dout, void* dq,
                         void* dk, void* dv, float* dg, void* db, void* dw,
                         void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_problem(p, "gdn2_chunk_bwd_intra");
  if (rc) return rc;
  if (!q || !k || !v || !g || !b || !w || !saved || !dout || !dq || !dk || !dv || !dg || !db || !dw)
    return fail(GDN2_ERR_INVALID, "gdn2_chunk_bwd_intra: null tensor pointer");
  SavedLayout L = layout_of(p);
  BwdLayout BL = bwd_layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_chunk_bwd_intra: saved buffer %zu < %zu bytes",
                saved_bytes, L.total);
  if (workspace_bytes < BL.total || (!workspace && BL.total))
    return fail(GDN2_ERR_WORKSPACE, "gdn2_chunk_bwd_intra: workspace %zu < %zu bytes",
                workspace_bytes, BL.total);
  if (p->seqs.n_chunks == 0) return GDN2_OK;
  rc = check_aligned16(p, "gdn2_chunk_bwd_intra",
                       {q, k, v, g, b, w, saved, dout, workspace, dq, dk, dv, dg, db, dw});
  if (rc) return rc;
  BwdIntraArgs a;
  a.seqs = make_seqs(p);
  a.H = p->H; a.K = p->K; a.V = p->V;
  a.scale = p->scale;
  a.l2norm = p->use_qk_l2norm;
  a.gate = gate_of(p);
  a.q = q; a.k = k; a.v = v; a.g = g; a.b = b; a.w = w;
  a.dout = dout;
  a.saved = static_cast<const unsigned char*>(saved);
  a.L = L;
  a.ws = static_cast<unsigned char*>(workspace);
  a.BL = BL;
  a.dq = dq; a.dk = dk; a.dv = dv; a.dg = dg; a.db = db; a.dw = dw;
  a.total_rows = p->seqs.total_tokens;
  cudaError_t e = fault_word(&a.fault);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_chunk_bwd_intra");
  e = bwd_intra_dispatch(p, a, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_chunk_bwd_intra");
}

int gdn2_chunk_bwd(const gdn2_chunk_problem* p, const void* q, const void* k, const void* v,
                   const float* g, const void* b, const void* w, const void* saved,
                   size_t saved_bytes, const void* dout, const float* dht, void* dq, void* dk,
                   void* dv, float* dg, void* db, void* dw, float* dh0, void* workspace,
                   size_t workspace_bytes, void* stream) {
  int rc = gdn2_chunk_bwd_state(p, saved, saved_bytes, dout, dht, dh0, workspace,
                                workspace_bytes, stream);
  if (rc) return rc;
  return gdn2_chunk_bwd_intra(p, q, k, v, g, b, w, saved, saved_bytes, dout, dq, dk, dv, dg, db,
                              dw, workspace, workspace_bytes, stream);
}

int gdn2_recurrent_fwd(const gdn2_recurrent_problem* p, const void* q, const void* k,
                       const void* v, const float* g, const void* b, const void* w,
                       const float* h0, void* o, float* ht, void* stream) {
  if (!p) return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: null problem");
  if (p->B <= 0 || p->T < 0 || p->H <= 0 || p->HV <= 0 || p->K <= 0 || p->V <= 0)
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: bad sizes B=%d T=%d H=%d HV=%d K=%d V=%d",
                p->B, p->T, p->H, p->HV, p->K, p->V);
  if (p->HV % p->H != 0)
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: HV=%d is not a multiple of H=%d", p->HV,
                p->H);
  if (p->K > 256 || p->V > 256)
    return fail(GDN2_ERR_UNSUPPORTED, "gdn2_recurrent_fwd: head sizes up to 256 are supported");
  if (!dtype_ok(p->dtype)) return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: unknown dtype");
  if (p->cu_seqlens && p->B != 1)
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: cu_seqlens requires B == 1 (got %d)", p->B);
  if (!p->cu_seqlens && p->n_seqs != p->B)
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: n_seqs (%d) must equal B (%d)", p->n_seqs,
                p->B);
  if (p->state_indices && p->state_stride < (int64_t)p->HV * p->K * p->V)
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: state_stride too small");
  if (p->state_indices_stride < 0 || (p->state_indices_stride > 0 && !p->state_indices))
    return fail(GDN2_ERR_INVALID,
                "gdn2_recurrent_fwd: state_indices_stride needs 2-D state_indices");
  if (p->num_accepted_tokens && p->state_indices_stride == 0)
    return fail(GDN2_ERR_INVALID,
                "gdn2_recurrent_fwd: num_accepted_tokens needs 2-D state_indices");
  if (p->gate < 0 || p->gate > 2 || (p->gate && !p->A_log))
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: gate %d needs A_log (modes 0..2)",
                p->gate);
  if (!q || !k || !v || !g || !b || !w || !o)
    return fail(GDN2_ERR_INVALID, "gdn2_recurrent_fwd: null tensor pointer");
  if (p->n_seqs == 0) return GDN2_OK;
  RecArgs a;
  a.B = p->B; a.T = p->T; a.H = p->H; a.HV = p->HV; a.K = p->K; a.V = p->V;
  a.scale = p->scale;
  a.l2norm = p->use_qk_l2norm;
  a.n_seqs = p->n_seqs;
  a.cu = p->cu_seqlens;
  a.state_idx = p->state_indices;
  a.state_stride = p->state_stride;
  a.idx_stride = p->state_indices_stride;
  a.n_accepted = p->num_accepted_tokens;
  a.A_log = p->A_log;
  a.dt_bias = p->dt_bias;
  a.gate = p->gate;
  a.lower_bound = p->lower_bound;
  a.q = q; a.k = k; a.v = v; a.g = g; a.b = b; a.w = w;
  a.h0 = h0; a.o = o; a.ht = ht;
  cudaError_t e = fault_word(&a.fault);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_recurrent_fwd");
  e = dispatch_rec(p->dtype, head_bucket(p->K, p->V), a, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_recurrent_fwd");
}

int gdn2_cp_fwd_prescan(const gdn2_chunk_problem* p, const void* saved, size_t saved_bytes,
                        float* hm, void* workspace, size_t workspace_bytes, void* stream) {
  (void)workspace;
  (void)workspace_bytes;
  int rc = check_problem(p, "gdn2_cp_fwd_prescan");
  if (rc) return rc;
  if (!saved || !hm) return fail(GDN2_ERR_INVALID, "gdn2_cp_fwd_prescan: null pointer");
  SavedLayout L = layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_cp_fwd_prescan: saved buffer too small");
  if (p->seqs.n_seqs == 0) return GDN2_OK;
  FwdStateArgs a;
  a.seqs = make_seqs(p);
  a.H = p->H; a.K = p->K; a.V = p->V;
  a.h0 = nullptr; a.o = nullptr; a.ht = nullptr;
  a.saved = static_cast<unsigned char*>(const_cast<void*>(saved));
  a.L = L;
  a.prescan = 1;
  a.hm = hm;
  cudaError_t e = fwd_state_dispatch(p, a, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_cp_fwd_prescan");
}

int gdn2_cp_bwd_prescan(const gdn2_chunk_problem* p, const void* saved, size_t saved_bytes,
                        const void* dout, const float* dht, float* dhm, void* workspace,
                        size_t workspace_bytes, void* stream) {
  int rc = check_problem(p, "gdn2_cp_bwd_prescan");
  if (rc) return rc;
  if (!saved || !dout || !dhm) return fail(GDN2_ERR_INVALID, "gdn2_cp_bwd_prescan: null pointer");
  SavedLayout L = layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_cp_bwd_prescan: saved buffer too small");
  if (p->seqs.n_seqs == 0) return GDN2_OK;
  BwdStateArgs s;
  s.seqs = make_seqs(p);
  s.H = p->H; s.K = p->K; s.V = p->V;
  s.dout = dout; s.dht = dht; s.dh0 = dhm;
  s.saved = static_cast<const unsigned char*>(saved);
  s.L = L;
  s.ws = nullptr;
  s.BL = bwd_layout_of(p);
  s.prescan = 1;
  s.total_rows = p->seqs.total_tokens;
  // With a workspace of gdn2_cp_workspace_bytes() the span-start gradient
  // comes from the tensor-core backward state pass (its dh0 output, dht as
  // the end gradient); the per-chunk dh / dVN tiles it also writes land in
  // the workspace and are not used.  Without one, the register-state pre-scan.
  const size_t need = gdn2_cp_workspace_bytes(p);
  if (workspace && need && workspace_bytes >= need) {
    BwdStateArgs t = s;
    t.ws = static_cast<unsigned char*>(workspace);
    t.prescan = 0;
    if (bwd_state_tc_ok(t, 1)) {
      cudaError_t e = launch_bwd_state_tc(t, (cudaStream_t)stream);
      return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_cp_bwd_prescan");
    }
  }
  cudaError_t e = bwd_state_dispatch(p, s, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_cp_bwd_prescan");
}

int gdn2_cp_merge(const gdn2_chunk_problem* p, const float* hm_all, const float* dhm_all,
                  int32_t rank, int32_t world, int32_t forward, const float* init,
                  float* state_out, void* stream) {
  int rc = check_problem(p, "gdn2_cp_merge");
  if (rc) return rc;
  if (world <= 0 || rank < 0 || rank >= world)
    return fail(GDN2_ERR_INVALID, "gdn2_cp_merge: rank %d outside world %d", rank, world);
  if (!hm_all || !state_out || (!forward && !dhm_all))
    return fail(GDN2_ERR_INVALID, "gdn2_cp_merge: null pointer");
  const int N = p->seqs.n_seqs;
  if (N == 0) return GDN2_OK;
  dim3 grid((p->V + 31) / 32, N * p->H);
  const uintptr_t al = reinterpret_cast<uintptr_t>(hm_all) | reinterpret_cast<uintptr_t>(dhm_all);
  if (p->K <= kMerge2MaxK && p->K % 16 == 0 && p->V % 4 == 0 && (al & 15) == 0) {
    const size_t smem = merge2_smem_bytes();
    cudaError_t e = cudaFuncSetAttribute(k_cp_merge2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return cuda_fail(e, "gdn2_cp_merge");
    k_cp_merge2<<<grid, kThreads, smem, (cudaStream_t)stream>>>(
        N, p->H, p->K, p->V, hm_all, dhm_all, rank, world, forward, init, state_out, nullptr);
    e = cudaGetLastError();
    return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_cp_merge");
  }
  const size_t smem = merge_smem_bytes(p->K);
  cudaError_t e = cudaFuncSetAttribute(k_cp_merge, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_cp_merge");
  k_cp_merge<<<grid, kThreads, smem, (cudaStream_t)stream>>>(N, p->H, p->K, p->V, hm_all, dhm_all,
                                                             rank, world, forward, init, state_out);
  e = cudaGetLastError();
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_cp_merge");
}

int gdn2_cp_unfold(const gdn2_chunk_problem* p, const float* hm_sub, const float* dhm_sub,
                   int32_t n_sub, int32_t forward, const float* init, float* states,
                   void* stream) {
  int rc = check_problem(p, "gdn2_cp_unfold");
  if (rc) return rc;
  if (n_sub <= 0) return fail(GDN2_ERR_INVALID, "gdn2_cp_unfold: %d sub-spans", n_sub);
  if (!hm_sub || !states || (!forward && !dhm_sub))
    return fail(GDN2_ERR_INVALID, "gdn2_cp_unfold: null pointer");
  const uintptr_t al = reinterpret_cast<uintptr_t>(hm_sub) | reinterpret_cast<uintptr_t>(dhm_sub);
  if (p->K > kMerge2MaxK || p->K % 16 != 0 || p->V % 4 != 0 || (al & 15) != 0)
    return fail(GDN2_ERR_UNSUPPORTED,
                "gdn2_cp_unfold: needs K <= 128 (a multiple of 16), V a multiple of 4 and "
                "16-byte aligned maps");
  const int N = p->seqs.n_seqs;
  if (N == 0) return GDN2_OK;
  dim3 grid((p->V + 31) / 32, N * p->H);
  const size_t smem = merge2_smem_bytes();
  cudaError_t e = cudaFuncSetAttribute(k_cp_merge2, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return cuda_fail(e, "gdn2_cp_unfold");
  k_cp_merge2<<<grid, kThreads, smem, (cudaStream_t)stream>>>(
      N, p->H, p->K, p->V, hm_sub, dhm_sub, forward ? n_sub - 1 : 0, n_sub, forward, init,
      nullptr, states);
  e = cudaGetLastError();
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_cp_unfold");
}

int gdn2_test_fwd_state_wait_timeout(const gdn2_chunk_problem* p, void* o, void* saved,
                                     size_t saved_bytes, int32_t skip_chunk, uint64_t wait_ns,
                                     void* stream) {
  int rc = check_problem(p, "gdn2_test_fwd_state_wait_timeout");
  if (rc) return rc;
  if (!o || !saved)
    return fail(GDN2_ERR_INVALID, "gdn2_test_fwd_state_wait_timeout: null o or saved");
  if (wait_ns == 0 || wait_ns > 1000000000ull)
    return fail(GDN2_ERR_INVALID,
                "gdn2_test_fwd_state_wait_timeout: wait_ns must be in 1 .. 1e9 (got %llu)",
                (unsigned long long)wait_ns);
  SavedLayout L = layout_of(p);
  if (saved_bytes < L.total)
    return fail(GDN2_ERR_WORKSPACE, "gdn2_test_fwd_state_wait_timeout: saved buffer too small");
  if (p->seqs.n_seqs == 0) return GDN2_OK;
  FwdStateArgs a;
  a.seqs = make_seqs(p);
  a.H = p->H; a.K = p->K; a.V = p->V;
  a.h0 = nullptr; a.o = o; a.ht = nullptr;
  a.saved = static_cast<unsigned char*>(saved);
  a.L = L;
  a.prescan = 0;
  a.hm = nullptr;
  a.wait_ns = wait_ns;
  a.skip_chunk = skip_chunk;
  if (!fwd_state_tc_ok(a, p->dtype == GDN2_DTYPE_BF16))
    return fail(GDN2_ERR_UNSUPPORTED,
                "gdn2_test_fwd_state_wait_timeout: only problems of the tcgen05 state pass "
                "(bf16, K = V = 128, 16-byte aligned buffers)");
  cudaError_t e = launch_fwd_state_tc(a, (cudaStream_t)stream);
  return e == cudaSuccess ? GDN2_OK : cuda_fail(e, "gdn2_test_fwd_state_wait_timeout");
}

int gdn2_fault_status(void* stream, int32_t clear) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) {
    cuda_fail(e, "gdn2_fault_status");
    return -1;
  }
  unsigned int bits = 0;
  e = read_fault_bits(&bits, clear != 0);
  if (e != cudaSuccess) {
    cuda_fail(e, "gdn2_fault_status");
    return -1;
  }
  return (int)(bits & 0x7fffffffu);
}

}  // extern "C"
