// common.cuh -- shared device/host helpers for the ennx_b200 sm_100a library.
//
// Status words, bounded waits, bf16 bit helpers, Philox4x32-10 noise and the
// inline-PTX wrappers for TMA, mbarriers and tcgen05 (TMEM + UMMA).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/ennx_b200.h"

namespace ennx {

// ---------------------------------------------------------------------------
// host-side error reporting (thread-local last error, never abort)
// ---------------------------------------------------------------------------
int32_t set_error(int32_t code, const char* fmt, ...);
int32_t check_cuda(cudaError_t e, const char* what);
#define ENNX_TRY(expr)                                 \
  do {                                                 \
    int32_t _st = (expr);                              \
    if (_st != ENNX_B200_OK) return _st;               \
  } while (0)
#define ENNX_CUDA(expr, what)                                          \
  do {                                                                 \
    cudaError_t _e = (expr);                                           \
    if (_e != cudaSuccess) return ::ennx::check_cuda(_e, what);        \
  } while (0)
#define ENNX_LAUNCH_CHECK(what)                 \
  do {                                          \
    ::ennx::note_launch(1);                     \
    ENNX_CUDA(cudaGetLastError(), what);        \
  } while (0)

// Device-side error word shared by every kernel of one process and device.
// Kernels write a nonzero code (ENNX_B200_TIMEOUT, ...) instead of trapping.
int* device_error_word();
// an additional per-device status word (static device memory) that
// consume_device_error also reads and clears
void register_status_word(int dev, int* word);
int32_t consume_device_error(cudaStream_t stream);  // synchronises `stream`

// Number of SMs of the current device (cached per device).
int sm_count();

// Launch accounting and optional CUDA-event profiling per kernel class.
void note_launch(int n = 1);
struct ProfScope {
  int slot;
  cudaStream_t stream;
  ProfScope(const char* cls, cudaStream_t s, double flops, double bytes);
  ~ProfScope();
};

// Per-device staging area for small per-call descriptor arrays (leaves,
// terms, status words).  Grows on demand; one per device; not thread-safe.
void* staging(size_t bytes);

// ---------------------------------------------------------------------------
// bf16 helpers -- exact bit formulas (round to nearest even) shared with the
// oracle, so that device and CPU produce identical bits.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ float bf16_to_f32(uint16_t v) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(((uint32_t)v) << 16);
#else
  uint32_t u = ((uint32_t)v) << 16; float f; memcpy(&f, &u, 4); return f;
#endif
}
// Round to nearest even.  For finite inputs the hardware conversion produces
// exactly the bits of the reference formula (bits + 0x7fff + lsb) >> 16
// (rust/crates/ennx/src/dense/bf16.rs:270-273), including overflow to inf.
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) { return __bfloat16_as_ushort(__float2bfloat16_rn(f)); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo (low half), .y = hi
  return *reinterpret_cast<uint32_t*>(&v);
}

// bf16x2 arithmetic with one RNE rounding of the exact result, and a
// streaming 16-byte global load that does not allocate in L1.
__device__ __forceinline__ uint4 ldg_stream_v4(const uint16_t* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_add(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

// splitmix64 finaliser of the seeded sign (rust/crates/ennx/src/dense.rs:428-433).
__host__ __device__ __forceinline__ uint64_t mix64(uint64_t x) {
  uint64_t v = x + 0x9e3779b97f4a7c15ull;
  v = (v ^ (v >> 30)) * 0xbf58476d1ce4e5b9ull;
  v = (v ^ (v >> 27)) * 0x94d049bb133111ebull;
  return v ^ (v >> 31);
}
// One BF16 ulp toward `positive`, staying finite (dense/bf16.rs:276-292).
__device__ __forceinline__ uint16_t bf16_next(uint16_t v, bool positive) {
  if ((v & 0x7fffu) == 0) return positive ? 1u : 0x8001u;
  bool grows = ((v & 0x8000u) == 0) == positive;
  uint16_t cand = grows ? (uint16_t)(v + 1u) : (uint16_t)(v - 1u);
  if ((cand & 0x7f80u) != 0x7f80u) return cand;
  return grows ? (uint16_t)(v - 1u) : (uint16_t)(v + 1u);
}

// ---------------------------------------------------------------------------
// Population noise: Philox4x32-10 (Salmon et al., SC'11) + Box-Muller.
// Element e of tensor t for antithetic pair p under population seed s is the
// (e % 8)-th normal of block e / 8: counter {lo(blk), hi(blk), t, p}, key
// {lo(s), hi(s)}; each of the four output words w gives one Box-Muller pair
// from its two 16-bit halves (radius from the low half, angle from the high).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0 = __umulhi(0xD2511F53u, c[0]);
    uint32_t lo0 = 0xD2511F53u * c[0];
    uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]);
    uint32_t lo1 = 0xCD9E8D57u * c[2];
    uint32_t n0 = hi1 ^ c[1] ^ k0;
    uint32_t n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// Box-Muller on the two 16-bit halves of one Philox word: u1 = (lo + 1/2) / 2^16
// lies in (0, 1) exactly (radius at most sqrt(2 ln 2^17) = 4.86), angle
// 2*pi*(hi / 2^16 - 1/2) in [-pi, pi).  Uses the SFU approximations (log2,
// rsqrt, sin/cos on [-pi, pi]); values agree with the fp64 oracle to ~1e-6.
__device__ __forceinline__ void box_muller16(uint32_t w, float& z0, float& z1) {
  const float u1 = __fmul_rn(__fadd_rn((float)(w & 0xffffu), 0.5f), 1.52587890625e-05f);
  const float u2 = __fmul_rn((float)(w >> 16), 1.52587890625e-05f);
  const float x = __fmul_rn(-1.3862943611198906f, __log2f(u1));  // -2 ln(u1) = -2 ln2 log2(u1) > 0
  const float r = x > 0.0f ? __fmul_rn(x, rsqrtf(x)) : 0.0f;
  float s, c;
  __sincosf(__fmul_rn(6.283185307179586f, __fsub_rn(u2, 0.5f)), &s, &c);
  z0 = __fmul_rn(r, c);
  z1 = __fmul_rn(r, s);
}

__device__ __forceinline__ void noise8(uint64_t seed, uint32_t pair, uint32_t tensor, uint64_t block, float z[8]) {
  uint32_t c[4] = {(uint32_t)block, (uint32_t)(block >> 32), tensor, pair};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
#pragma unroll
  for (int j = 0; j < 4; ++j) box_muller16(c[j], z[2 * j], z[2 * j + 1]);
}

// ---------------------------------------------------------------------------
// bounded waits: ~2 s of globaltimer, then record ENNX_B200_TIMEOUT and give up
// ---------------------------------------------------------------------------
constexpr unsigned long long kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Returns false (and records a timeout) if the phase does not complete in time.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 255u) == 0 && globaltimer() - t0 > kWaitLimitNs) {
      if (err) atomicExch(err, ENNX_B200_TIMEOUT);
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Pair (cta_group::2) form: the loaded bytes complete on the mbarrier at the
// shared::cluster address `bar_cluster` (the leader CTA's barrier).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"((uint64_t)map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same smem location in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16, single CTA.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A * B^T over a CTA pair: M = 256 (128 rows of A in each CTA), B's N
// rows split in halves between the two CTAs.  Issued by the leader CTA.
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on the barrier at this smem offset in every CTA of `mask` when
// the pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                     // D format f32
         | (1u << 7)                   // A format bf16
         | (1u << 10)                  // B format bf16
         | ((uint32_t)(N >> 3) << 17)  // N / 8
         | ((uint32_t)(M >> 4) << 24); // M / 16
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row groups 1024 B apart (SBO), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// K-major, 64-byte swizzle: rows of 64 B (32 bf16), 8-row groups 512 B apart.
__device__ __forceinline__ uint64_t smem_desc_sw64(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(512u >> 4) << 32) |
         ((uint64_t)1u << 46) | ((uint64_t)4u << 61);
}

// MN-major operand (rows of 64 MN-contiguous bf16 = 128 B, 128-byte swizzle):
// SBO = 1024 B between groups of 8 K-rows, LBO = byte distance between
// consecutive 64-wide MN blocks.
__device__ __forceinline__ uint64_t smem_desc_sw128_mn(uint32_t saddr, uint32_t lbo_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)(1024u >> 4) << 32) | ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}

// 32 lanes x 32 columns of 32-bit TMEM words -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// 32 lanes x 32 columns of 32-bit TMEM words <- 32 registers per thread.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// ---------------------------------------------------------------------------
// host: tensor-map encoding through the driver entry point (no -lcuda)
// ---------------------------------------------------------------------------
int32_t make_tmap_2d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                          uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer, bool swizzle128);
// swizzle_bytes: 0 (none), 32, 64 or 128
int32_t make_tmap_2d_bf16_sw(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                             uint64_t row_stride_elems, uint32_t box_inner, uint32_t box_outer, int swizzle_bytes);

}  // namespace ennx
