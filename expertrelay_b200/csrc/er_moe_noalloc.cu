// er_moe_noalloc.cu -- er_moe_block_noalloc: the MoE block for callers that
// cannot allocate device memory.
//
// Some hosts of this library have no way to call cudaMalloc for a
// workspace: a serving runtime whose memory manager has already claimed all
// of HBM for its expert cache and KV pages, or a foreign-language binding
// (cgo, JNI, a plain C plugin) that runs without a device allocator of its
// own. For them the block's scratch lives in a fixed array compiled into
// this file, so a call needs only its inputs and outputs.
//
// Contract:
//  * the scratch is kMoeNoallocScratchBytes (8 MiB) of device memory per GPU,
//    held from the first call on that GPU until the process exits; a batch
//    whose workspace (er_moe_workspace_bytes) exceeds it is rejected with
//    ER_ENOSPACE before anything is launched (at Qwen1.5-MoE-A2.7B shapes:
//    up to 96 tokens per call on the GEMV / SIMT GEMM paths, 64 on the
//    tensor-core path, whose int8 operand slices take room too);
//  * the first call on a device looks up the array's device address (once
//    per device, with that device current) and caches it; make that first
//    call before any stream capture;
//  * every call on a device shares the one array and it keeps the previous
//    call's contents; the block writes every scratch byte it reads before
//    reading it, so nothing has to start at zero, but calls that overlap on
//    the GPU (other streams, other threads) race on the array and must be
//    serialised by the caller;
//  * it calls no cudaMalloc, cudaFree or allocating library routine.
#include <mutex>

#include "er_internal.cuh"

namespace {

constexpr size_t kMoeNoallocScratchBytes = size_t(8) << 20;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_moe_scratch[kMoeNoallocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_moe_scratch on the current device. In host code the
// symbol only names a host-side stand-in; the real address comes from
// cudaGetSymbolAddress with the device current.
int scratch_address(void** out) {
  int dev = 0;
  if (int rc = er::cuda_check(cudaGetDevice(&dev), "cudaGetDevice")) return rc;
  if (dev < 0 || dev >= kMaxDevices)
    return er::fail(ER_EINVAL, "er_moe_block_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (int rc = er::cuda_check(cudaGetSymbolAddress(&p, g_moe_scratch), "cudaGetSymbolAddress(scratch)")) return rc;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return ER_OK;
}

}  // namespace

extern "C" int er_moe_block_noalloc(const er_moe_weights* w, const er_moe_io* io, void* stream) {
  using namespace er;
  if (w && io && io->n > 0) {
    const size_t need = er_moe_workspace_bytes(w, io->n, io->path);
    if (need > kMoeNoallocScratchBytes)
      return fail(ER_ENOSPACE,
                  "er_moe_block_noalloc: %d tokens need %zu bytes of scratch; the fixed scratch holds %zu bytes "
                  "(split the batch, or use er_moe_block with a caller workspace)",
                  io->n, need, kMoeNoallocScratchBytes);
  }
  void* scratch = nullptr;
  if (int rc = scratch_address(&scratch)) return rc;
  return er_moe_block(w, io, scratch, kMoeNoallocScratchBytes, stream);
}
