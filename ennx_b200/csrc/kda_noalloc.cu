// kda_noalloc.cu -- chunked KDA for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc: code running inside a CUDA graph that
// is being captured (allocation is not a capturable operation), hosts that
// pre-reserve every byte of device memory for their own pool and forbid other
// allocations, and embedders (JAX/XLA custom calls, game engines, real-time
// loops) where an allocation in the hot path means an unbounded stall.  The
// regular ennx_b200_kda_chunked needs a caller-provided workspace for its
// per-chunk operand records; this variant takes that scratch from one
// file-scope device array instead, so it allocates nothing at all.
//
// The array is a fixed kNoAllocScratchBytes (32 MiB) on every GPU that loads
// this library, held until the process exits.  That bounds the problem size:
// batch * heads * ceil(seq / 64) chunk records of 66 048 bytes each, i.e. up
// to 508 (sequence, head, chunk) triples -- for example one 2048-token
// sequence with 16 heads.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace ennx {
namespace {

constexpr size_t kNoAllocScratchBytes = 32ull << 20;

// Device scratch shared by every call on a device.  Host code must not use
// the symbol as an address: it is a host-side stand-in; the device address
// comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_kda_scratch[kNoAllocScratchBytes];

// This path's own status word: a bounded device wait that gives up writes
// ENNX_B200_TIMEOUT here (the regular entry points use a word that is
// allocated on first use, which this path must not do).  Zero-initialised at
// module load; ennx_b200_device_status reads and clears it.
static __device__ int g_kda_noalloc_status;

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices];
int* g_status_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Resolve the device addresses of the scratch array and of the status word
// once per device, with that device current.  The first call on a device
// therefore runs this set-up and should happen before any stream capture
// begins.
int32_t scratch_address(void** out, int** status) {
  int dev = 0;
  ENNX_CUDA(cudaGetDevice(&dev), "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return set_error(ENNX_B200_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_kda_scratch);
    if (e != cudaSuccess || !p) return check_cuda(e, "cudaGetSymbolAddress(kda scratch)");
    void* w = nullptr;
    e = cudaGetSymbolAddress(&w, g_kda_noalloc_status);
    if (e != cudaSuccess || !w) return check_cuda(e, "cudaGetSymbolAddress(kda status word)");
    g_scratch_ptr[dev] = p;
    g_status_ptr[dev] = (int*)w;
    register_status_word(dev, (int*)w);
  }
  *out = g_scratch_ptr[dev];
  *status = g_status_ptr[dev];
  return ENNX_B200_OK;
}

}  // namespace
}  // namespace ennx

extern "C" int32_t ennx_b200_kda_chunked_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                                 const float* g, const float* beta, float* state, uint16_t* o,
                                                 int32_t batch, int32_t seq, int32_t heads, void* stream) {
  using namespace ennx;
  if (!q || !k || !v || !g || !beta || !o) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_noalloc: null argument");
  if (batch <= 0 || seq <= 0 || heads <= 0) return set_error(ENNX_B200_INVALID_ARGUMENT, "kda_noalloc: empty input");
  const size_t need = kda_workspace_bytes(batch, seq, heads);
  if (need > kNoAllocScratchBytes)
    return set_error(ENNX_B200_INVALID_ARGUMENT,
                     "kda_noalloc: batch*heads*ceil(seq/64) chunks need %zu bytes of scratch, the static scratch "
                     "holds %zu; use ennx_b200_kda_chunked with a caller workspace",
                     need, kNoAllocScratchBytes);
  void* scratch = nullptr;
  int* status = nullptr;
  ENNX_TRY(scratch_address(&scratch, &status));
  return launch_kda_chunked(q, k, v, (long long)heads * 128, g, beta, state, o, (long long)heads * 128, batch, seq,
                            heads, scratch, kNoAllocScratchBytes, (cudaStream_t)stream, nullptr, status);
}
