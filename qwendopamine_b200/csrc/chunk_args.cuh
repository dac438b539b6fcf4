// chunk_args.cuh -- argument blocks passed by value to the GDN-2 kernels.
// Shared by the kernel translation units and the C-ABI layer (abi.cu).
#pragma once

#include "common.cuh"

namespace gdn2 {

// Gate in kernel: the raw g becomes the log-decay -exp(A_log[h]) *
// softplus(g + dt_bias[h][k]) (mode 1) or lower_bound * sigmoid(exp(A_log[h])
// * (g + dt_bias[h][k])) (mode 2); mode 0 takes g as it is.
struct GateArgs {
  const float* A_log;
  const float* dt_bias;
  int mode;
  float lower_bound;
  float* dA_log;    // backward: += dL/dA_log [H]
  float* ddt_bias;  // backward: += dL/d dt_bias [H*K] or null
};

// Log-decay from the raw gate input g of head h, channel c.
__device__ __forceinline__ float gate_apply(const GateArgs& gt, float g, int h, int c, int K) {
  const float x = gt.dt_bias ? g + gt.dt_bias[h * K + c] : g;
  const float A = expf(gt.A_log[h]);
  if (gt.mode == 2) return gt.lower_bound / (1.f + expf(-A * x));
  return -A * (x > 20.f ? x : log1pf(expf(x)));
}

// Backward of gate_apply (the reference's kda_gate_bwd): from dyg, the
// gradient of the log-decay, the gradient of the raw input (returned) and the
// term this element adds to dL/dA_log (*dA).
__device__ __forceinline__ float gate_grad(const GateArgs& gt, float g, float dyg, int h, int c,
                                           int K, float* dA) {
  const float x = gt.dt_bias ? g + gt.dt_bias[h * K + c] : g;
  const float A = expf(gt.A_log[h]);
  if (gt.mode == 2) {
    const float sig = 1.f / (1.f + expf(-A * x));
    const float dg = dyg * gt.lower_bound * sig * (1.f - sig) * A;
    *dA = dg * x;
    return dg;
  }
  const float sig = 1.f / (1.f + expf(-x));
  *dA = dyg * (-A * (x > 20.f ? x : log1pf(expf(x))));
  return -A * dyg * sig;
}

struct FwdIntraArgs {
  Seqs seqs;
  int H, K, V;
  float scale;
  int l2norm;
  GateArgs gate;
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const void* b;
  const void* w;
  unsigned char* saved;
  SavedLayout L;
  unsigned int* fault;  // device fault word (bounded waits that ran out)
  int64_t total_rows;   // token rows of q, k, v, g, b, w (bounds of their TMA views)
  int max_ctas = 0;     // persistent kernel: at most this many CTAs (0: one per SM)
};

struct FwdStateArgs {
  Seqs seqs;
  int H, K, V;
  const float* h0;   // [N,H,K,V] or null
  void* o;           // [rows,H,V] or null (pre-scan)
  float* ht;         // [N,H,K,V] or null
  unsigned char* saved;
  SavedLayout L;
  // pre-scan mode: carry [h | M] over V+K columns from [0 | I]; write hm.
  int prescan;
  float* hm;         // [N,H,K,V+K]
  // Test of the bounded-wait abort path (tcgen05 pass only): every mbarrier
  // wait gives up after wait_ns (0: the built-in limit) and chunk
  // skip_chunk's tiles are never requested (-1: none).
  uint64_t wait_ns = 0;
  int skip_chunk = -1;
  int max_ctas = 0;  // tcgen05 pass: the value-half split only within this many CTAs (0: SMs)
};

struct BwdStateArgs {
  Seqs seqs;
  int H, K, V;
  const void* dout;   // [rows,H,V]
  const float* dht;   // [N,H,K,V] or null
  float* dh0;         // [N,H,K,V] or null
  const unsigned char* saved;
  SavedLayout L;
  unsigned char* ws;
  BwdLayout BL;
  int prescan;        // 1: write nothing per chunk, only the span-start gradient
  int64_t total_rows; // token rows of dout (bounds of its TMA view)
  int max_ctas = 0;   // tcgen05 pass: the value-half split only within this many CTAs (0: SMs)
};

struct BwdIntraArgs {
  Seqs seqs;
  int H, K, V;
  float scale;
  int l2norm;
  GateArgs gate;
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const void* b;
  const void* w;
  const void* dout;
  const unsigned char* saved;
  SavedLayout L;
  unsigned char* ws;   // dh, dVN (read); the wide kernels' fp32 dq / dk rows (written)
  BwdLayout BL;
  void* dq;
  void* dk;
  void* dv;
  float* dg;
  void* db;
  void* dw;
  unsigned int* fault;  // device fault word (bounded waits that ran out)
  int64_t total_rows;   // token rows of q, k, v, g, b, w, dout (bounds of their TMA views)
};

struct RecArgs {
  int B, T, H, HV, K, V;
  float scale;
  int l2norm;
  int n_seqs;
  const int32_t* cu;         // [N+1] or null
  const int32_t* state_idx;  // [N] or [N][idx_stride] or null
  int64_t state_stride;
  int64_t idx_stride;        // > 0: speculative decoding, a state slot per token
  const int32_t* n_accepted; // [N] or null (speculative decoding)
  const float* A_log;        // [H] (gate in kernel)
  const float* dt_bias;      // [H*K] or null
  int gate;                  // 0: g is the log-decay; 1: softplus gate; 2: lower-bound gate
  float lower_bound;
  const void* q;
  const void* k;
  const void* v;
  const float* g;
  const void* b;
  const void* w;
  const float* h0;
  void* o;
  float* ht;
  unsigned int* fault;  // device fault word (bounded waits that ran out)
};

}  // namespace gdn2
