// noalloc.cu -- chunkwise backward that allocates nothing.
//
// gdn2_chunk_bwd needs a scratch workspace (per-chunk state gradients and dVN,
// gdn2_chunk_bwd_workspace_bytes()) that the caller normally allocates.  Some
// callers cannot allocate device memory when they run the backward: a plugin
// host that owns all device memory and hands an op only its planned inputs and
// outputs, or a serving / training loop that has reserved nearly all HBM up
// front and must not risk an allocation failure, or the implicit device-wide
// synchronisation that cudaMalloc / cudaFree can cause, in the middle of a step.
// gdn2_chunk_bwd_noalloc serves them: its scratch is the file-scope array
// below, which every GPU that loads this library holds until the process exits.
//
// * Size limit: GDN2_NOALLOC_SCRATCH_BYTES (32 MiB).  A problem whose workspace
//   is larger is rejected with GDN2_ERR_WORKSPACE and a message giving both
//   sizes.  (bf16, K = V = 128: 48 KiB per (chunk, head), so 682 chunk-heads,
//   e.g. one 2,688-token sequence with 16 heads.)
// * Set-up: the first call on a device, with that device current, looks the
//   array's device address up once (cudaGetSymbolAddress) and caches it; make
//   that first call before any stream capture on that device.  The cache is
//   kept per device for the life of the process: after cudaDeviceReset (or
//   anything else that destroys and re-creates the device's primary context)
//   the cached address is stale, so a process that resets a device must not
//   call this entry point on it again.
// * Sharing: every call on a device uses the same array and leaves its
//   contents behind.  Nothing in it has to start at zero -- the reverse state
//   pass writes every byte the per-chunk pass later reads -- so it is never
//   cleared.  Calls whose work overlaps on the GPU (other streams, other host
//   threads) race on the array: order them.
#include <cstdio>
#include <mutex>

#include "../../include/gdn2_b200.h"
#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[GDN2_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (set up once).
int scratch_for_current_device(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return 0;
}

}  // namespace

namespace gdn2 {
int set_error(int code, const char* msg);
}

extern "C" int gdn2_chunk_bwd_noalloc(const gdn2_chunk_problem* p, const void* q, const void* k,
                                      const void* v, const float* g, const void* b, const void* w,
                                      const void* saved, size_t saved_bytes, const void* dout,
                                      const float* dht, void* dq, void* dk, void* dv, float* dg,
                                      void* db, void* dw, float* dh0, void* stream) {
  const size_t need = gdn2_chunk_bwd_workspace_bytes(p);
  if (need == 0) {
    // an invalid problem (gdn2_chunk_bwd reports why) or one with no chunks
    return gdn2_chunk_bwd(p, q, k, v, g, b, w, saved, saved_bytes, dout, dht, dq, dk, dv, dg, db,
                          dw, dh0, nullptr, 0, stream);
  }
  char msg[256];
  if (need > (size_t)GDN2_NOALLOC_SCRATCH_BYTES) {
    snprintf(msg, sizeof(msg),
             "gdn2_chunk_bwd_noalloc: this problem needs %zu bytes of scratch; the built-in "
             "scratch holds %zu (GDN2_NOALLOC_SCRATCH_BYTES) -- use gdn2_chunk_bwd with a "
             "caller-owned workspace",
             need, (size_t)GDN2_NOALLOC_SCRATCH_BYTES);
    return gdn2::set_error(GDN2_ERR_WORKSPACE, msg);
  }
  void* scratch = nullptr;
  int e = scratch_for_current_device(&scratch);
  if (e != 0) {
    snprintf(msg, sizeof(msg), "gdn2_chunk_bwd_noalloc: scratch set-up failed: CUDA error %d (%s)",
             e, cudaGetErrorString((cudaError_t)e));
    return gdn2::set_error(GDN2_ERR_CUDA, msg);
  }
  return gdn2_chunk_bwd(p, q, k, v, g, b, w, saved, saved_bytes, dout, dht, dq, dk, dv, dg, db, dw,
                        dh0, scratch, GDN2_NOALLOC_SCRATCH_BYTES, stream);
}
