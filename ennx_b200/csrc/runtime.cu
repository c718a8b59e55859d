// runtime.cu -- error reporting, device bookkeeping and tensor-map encoding.
#include <cudaTypedefs.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace ennx {

static thread_local std::string g_last_error;

int32_t set_error(int32_t code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int32_t check_cuda(cudaError_t e, const char* what) {
  return set_error(ENNX_B200_CUDA_ERROR, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

static constexpr int kMaxDevices = 64;
static std::mutex g_mu;
static int* g_err_word[kMaxDevices];
static int g_sms[kMaxDevices];

static int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int* device_error_word() {
  int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_err_word[d]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    cudaMemset(p, 0, sizeof(int));
    g_err_word[d] = p;
  }
  return g_err_word[d];
}

static int* g_extra_word[kMaxDevices];

void register_status_word(int dev, int* word) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (dev >= 0 && dev < kMaxDevices) g_extra_word[dev] = word;
}

// Reads and clears every status word of the current device: the shared word
// of the regular entry points (only if it exists already: a word that was
// never allocated was never written, so checking allocates nothing) and the
// static word of the allocation-free entry point.
int32_t consume_device_error(cudaStream_t stream) {
  int d = current_device();
  int* words[2];
  {
    std::lock_guard<std::mutex> lk(g_mu);
    words[0] = g_err_word[d];
    words[1] = g_extra_word[d];
  }
  ENNX_CUDA(cudaStreamSynchronize(stream), "stream synchronize");
  int worst = 0;
  for (int* w : words) {
    if (!w) continue;
    int host = 0;
    ENNX_CUDA(cudaMemcpy(&host, w, sizeof(int), cudaMemcpyDeviceToHost), "read device error word");
    if (host != 0) {
      ENNX_CUDA(cudaMemset(w, 0, sizeof(int)), "clear device error word");
      if (!worst) worst = host;
    }
  }
  if (worst == ENNX_B200_TIMEOUT)
    return set_error(ENNX_B200_TIMEOUT, "a device wait exceeded its bound; the kernel returned early");
  if (worst) return set_error(worst, "device kernel reported status %d", worst);
  return ENNX_B200_OK;
}

static void* g_stage[kMaxDevices];
static size_t g_stage_bytes[kMaxDevices];

void* staging(size_t bytes) {
  int d = current_device();
  if (g_stage_bytes[d] < bytes) {
    if (g_stage[d]) {
      cudaDeviceSynchronize();
      cudaFree(g_stage[d]);
    }
    size_t cap = bytes < 4096 ? 4096 : bytes * 2;
    g_stage[d] = nullptr;
    g_stage_bytes[d] = 0;
    if (cudaMalloc(&g_stage[d], cap) != cudaSuccess) return nullptr;
    g_stage_bytes[d] = cap;
  }
  return g_stage[d];
}

int sm_count() {
  int d = current_device();
  if (g_sms[d] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 148;
  }
  return g_sms[d];
}

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int32_t make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
  return make_tmap_2d_bf16_sw(map, base, inner, outer, row_stride_elems, box_inner, box_outer, swizzle128 ? 128 : 0);
}

int32_t make_tmap_2d_bf16_sw(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                             uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer, int swizzle_bytes) {
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    ENNX_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q),
              "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (q != cudaDriverEntryPointSuccess || !fn)
      return set_error(ENNX_B200_CUDA_ERROR, "cuTensorMapEncodeTiled is not available from the driver");
    g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
  }
  if (((uintptr_t)base & 15u) != 0 || (row_stride_elems * 2) % 16 != 0)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "TMA operand must be 16-byte aligned with a 16-byte row stride");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                        : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                        : swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                              : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(ENNX_B200_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d) for %llux%llu box %ux%u",
                     (int)r, (unsigned long long)inner, (unsigned long long)outer, box_inner, box_outer);
  return ENNX_B200_OK;
}

static std::atomic<uint64_t> g_launches{0};
void note_launch(int n) { g_launches.fetch_add((uint64_t)n, std::memory_order_relaxed); }

struct ProfClass {
  std::string name;
  int64_t launches = 0;
  double flops = 0, bytes = 0;
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> events;
};
static thread_local bool g_prof_on = false;
static thread_local std::vector<ProfClass> g_prof;
static thread_local std::vector<cudaEvent_t> g_event_pool;

static cudaEvent_t take_event() {
  if (!g_event_pool.empty()) {
    cudaEvent_t e = g_event_pool.back();
    g_event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

ProfScope::ProfScope(const char* cls, cudaStream_t s, double flops, double bytes) : slot(-1), stream(s) {
  if (!g_prof_on) return;
  for (size_t i = 0; i < g_prof.size(); ++i)
    if (g_prof[i].name == cls) slot = (int)i;
  if (slot < 0) {
    g_prof.push_back(ProfClass());
    g_prof.back().name = cls;
    slot = (int)g_prof.size() - 1;
  }
  ProfClass& c = g_prof[slot];
  c.launches += 1;
  c.flops += flops;
  c.bytes += bytes;
  cudaEvent_t a = take_event(), b = take_event();
  cudaEventRecord(a, s);
  c.events.push_back({a, b});
}

ProfScope::~ProfScope() {
  if (slot < 0 || !g_prof_on) return;
  cudaEventRecord(g_prof[slot].events.back().second, stream);
}

}  // namespace ennx

extern "C" {

uint64_t ennx_b200_launch_count(void) { return ennx::g_launches.load(); }

int32_t ennx_b200_profile_begin(void) {
  for (auto& c : ennx::g_prof)
    for (auto& e : c.events) { ennx::g_event_pool.push_back(e.first); ennx::g_event_pool.push_back(e.second); }
  ennx::g_prof.clear();
  ennx::g_prof_on = true;
  return ENNX_B200_OK;
}

int32_t ennx_b200_profile_end(ennx_b200_profile_entry* out, int32_t max_entries, int32_t* num_entries) {
  ennx::g_prof_on = false;
  ENNX_CUDA(cudaDeviceSynchronize(), "profile sync");
  int32_t n = 0;
  for (auto& c : ennx::g_prof) {
    double ms = 0;
    for (auto& e : c.events) {
      float t = 0;
      if (cudaEventElapsedTime(&t, e.first, e.second) == cudaSuccess) ms += t;
    }
    if (out && n < max_entries) {
      memset(&out[n], 0, sizeof(out[n]));
      strncpy(out[n].name, c.name.c_str(), sizeof(out[n].name) - 1);
      out[n].launches = c.launches;
      out[n].total_ms = ms;
      out[n].flops = c.flops;
      out[n].bytes = c.bytes;
    }
    ++n;
  }
  if (num_entries) *num_entries = n;
  return ENNX_B200_OK;
}

uint32_t ennx_b200_abi_version(void) { return ENNX_B200_ABI_VERSION; }

const char* ennx_b200_last_error(void) { return ennx::g_last_error.c_str(); }

int32_t ennx_b200_device_check(void) {
  int d = 0;
  ENNX_CUDA(cudaGetDevice(&d), "cudaGetDevice");
  cudaDeviceProp p;
  ENNX_CUDA(cudaGetDeviceProperties(&p, d), "cudaGetDeviceProperties");
  if (p.major != 10 || p.minor != 0)
    return ennx::set_error(ENNX_B200_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", d,
                           p.major, p.minor);
  return ENNX_B200_OK;
}

int32_t ennx_b200_device_status(void* stream) { return ennx::consume_device_error((cudaStream_t)stream); }

}  // extern "C"
