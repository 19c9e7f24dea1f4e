// Shared constants and small device helpers of the PESQ engine (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Phase timing of the kernels.  A build with -DPESQ_PHASE_PROBE records
// clock64() at each PESQ_STAMP(table, i) of the first and the last CTA of a
// launch (slots i and 8 + i of a 16-entry table defined by
// PESQ_PHASE_TABLE(table), readable from the host through the extern "C"
// function table_read); each stamp is preceded by a CTA barrier.  In a normal
// build both macros expand to nothing.
#ifdef PESQ_PHASE_PROBE
#define PESQ_PHASE_TABLE(name)                                                  \
  __device__ unsigned long long name[16];                                       \
  extern "C" int name##_read(unsigned long long* host) {                        \
    return (int)cudaMemcpyFromSymbol(host, name, sizeof(unsigned long long) * 16); \
  }
#define PESQ_STAMP(name, i)                                                          \
  do {                                                                               \
    __syncthreads();                                                                 \
    if (threadIdx.x == 0 && (blockIdx.x == 0 || blockIdx.x == gridDim.x - 1))        \
      name[(blockIdx.x ? 8 : 0) + (i)] = clock64();                                  \
  } while (0)
// PESQ_SPAN(table, i) brackets a whole kernel on the global nanosecond timer:
// slot i keeps the earliest CTA start, slot 8 + i the latest CTA end (the
// host zeroes the table, then reads it, through table_read / table_clear).
#define PESQ_SPAN_TABLE(name)                                                        \
  __device__ unsigned long long name[16];                                            \
  extern "C" int name##_read(unsigned long long* host) {                             \
    return (int)cudaMemcpyFromSymbol(host, name, sizeof(unsigned long long) * 16);   \
  }                                                                                  \
  extern "C" int name##_clear() {                                                    \
    unsigned long long init[16];                                                     \
    for (int i = 0; i < 16; ++i) init[i] = i < 8 ? ~0ull : 0ull;                     \
    return (int)cudaMemcpyToSymbol(name, init, sizeof(init));                        \
  }
__device__ __forceinline__ unsigned long long pesq_globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
#define PESQ_SPAN_BEGIN(name, i) \
  do {                           \
    if (threadIdx.x == 0) atomicMin(&name[(i)], pesq_globaltimer()); \
  } while (0)
#define PESQ_SPAN_END(name, i)                                                \
  do {                                                                        \
    __syncthreads();                                                          \
    if (threadIdx.x == 0) atomicMax(&name[8 + (i)], pesq_globaltimer());      \
  } while (0)
// Per-CTA start / end on the global timer (CTA b: slots 2b, 2b + 1), for up
// to 4096 CTAs of one kernel.
#define PESQ_CTA_TABLE(name)                                                         \
  __device__ unsigned long long name[8192];                                          \
  extern "C" int name##_read(unsigned long long* host) {                             \
    return (int)cudaMemcpyFromSymbol(host, name, sizeof(unsigned long long) * 8192); \
  }
#define PESQ_CTA_BEGIN(name) \
  do {                       \
    if (threadIdx.x == 0 && blockIdx.x < 4096) name[2 * blockIdx.x] = pesq_globaltimer(); \
  } while (0)
#define PESQ_CTA_END(name)                                                                    \
  do {                                                                                        \
    __syncthreads();                                                                          \
    if (threadIdx.x == 0 && blockIdx.x < 4096) name[2 * blockIdx.x + 1] = pesq_globaltimer(); \
  } while (0)
#else
#define PESQ_CTA_TABLE(name)
#define PESQ_CTA_BEGIN(name) \
  do {                       \
  } while (0)
#define PESQ_CTA_END(name) \
  do {                     \
  } while (0)
#define PESQ_PHASE_TABLE(name)
#define PESQ_STAMP(name, i) \
  do {                      \
  } while (0)
#define PESQ_SPAN_TABLE(name)
#define PESQ_SPAN_BEGIN(name, i) \
  do {                           \
  } while (0)
#define PESQ_SPAN_END(name, i) \
  do {                         \
  } while (0)
#endif

namespace pesq {

// ---------------------------------------------------------------------------
// geometry of the streaming kernels
// ---------------------------------------------------------------------------

// Threads of the streaming (front / back / iir) kernels; each thread owns one
// chunk of the covered span.
constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
// Samples per thread chunk.  33 is coprime with the 32 shared memory banks, so
// the stride-33 per-thread walks over a linearly staged span never conflict.
constexpr int kChunk = 33;
// Kogge-Stone doubling levels of the in-CTA state scan: the state handed to a
// chunk accounts for the previous kHorizonChunks chunks exactly and drops
// A^(kChunk * kHorizonChunks), whose norm the host checks (< 1e-11).
constexpr int kLevels = 5;
constexpr int kHorizonChunks = 1 << kLevels;
constexpr int kHorizon = kChunk * kHorizonChunks;  // 1056 samples
constexpr int kSpan = kThreads * kChunk;           // 16896 samples per CTA

// STFT of the PESQ model: 512-point frames, hop 256, 256 usable bins.
constexpr int kNfft = 512;
constexpr int kHop = 256;
constexpr int kBins = 256;
constexpr int kMaxBands = 64;

// Largest state size of a filter handled by the chunked scan.
constexpr int kMaxStates = 16;

// ---------------------------------------------------------------------------
// small helpers
// ---------------------------------------------------------------------------

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Linear fade of the first and last 15 samples of a row, applied as
// (value * head) * tail in that order; both factors are 1 outside their ramp.
// Mirrors the two sequential in-place products of torch_pesq/loss.py:163-165.
__device__ __forceinline__ float edge_ramp(float v, int64_t n, int64_t len) {
  const float head = n < 15 ? (float)(n + 1) * 0.0625f : 1.0f;
  const float tail = n >= len - 15 ? (float)(len - n) * 0.0625f : 1.0f;
  return (v * head) * tail;
}

// ---------------------------------------------------------------------------
// thread block cluster primitives (distributed shared memory)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}

// Full cluster barrier with release/acquire semantics on shared::cluster.
// Cluster-wide barrier.  The release / acquire pair orders every memory
// access of the arriving threads (shared, distributed shared and global)
// before the accesses of all cluster threads after the wait, so values that
// one CTA writes to global memory before the barrier are read by the other
// CTAs of its cluster after it (through L2, ld.global.cg) without a fence.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n"
               "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of `ptr` (a shared memory variable of this CTA) in the shared
// memory window of cluster rank `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(const void* ptr, uint32_t rank) {
  uint32_t local = (uint32_t)__cvta_generic_to_shared(ptr);
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}

__device__ __forceinline__ float dsmem_ld_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ double dsmem_ld_f64(uint32_t addr) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(addr) : "memory");
  return v;
}

__device__ __forceinline__ void dsmem_st_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

// Hardware base-2 exponential and logarithm (ex2.approx / lg2.approx, about
// 2^-22 relative error), for quantities whose use tolerates it.
__device__ __forceinline__ float exp2f_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float log2f_fast(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------

// A kernel launched with programmatic stream serialisation may start before
// the kernel preceding it on the stream has ended.  pdl_trigger() allows the
// kernel following this one to start (once every CTA of this grid has called
// it or exited); pdl_wait() blocks until the preceding kernel has completed and
// its memory is visible, and is a no-op in a kernel launched normally.  The
// chain kernels and the back kernel are launched this way and released at
// the end of their predecessors' CTAs (their table copies overlap the
// predecessor's tail; everything else waits in pdl_wait); the align kernel is
// released at the start of the chain adjoint and runs beside it.  Every
// kernel launched this way calls pdl_wait() before it exits, so its
// completion implies the completion of everything before it on the stream.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------------------
// global -> shared staging
// ---------------------------------------------------------------------------

static_assert(kSpan % kThreads == 0, "a span is a whole number of rows of the CTA");

// dst[i] = src[base + i] for i in [0, NT * kChunk), 0 where base + i lies
// outside [0, n).  Every thread issues all of its loads before its first
// shared store, so the whole span is in flight at once instead of one DRAM
// round trip per loop iteration.  Must be called by all NT threads of the CTA.
template <int NT = kThreads>
__device__ __forceinline__ void stage_span(float* dst, const float* src, int64_t base, int64_t n) {
  constexpr int kPer = kChunk;
  float v[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int64_t g = base + threadIdx.x + k * NT;
    v[k] = (g >= 0 && g < n) ? __ldg(src + g) : 0.0f;
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k) dst[threadIdx.x + k * NT] = v[k];
}

// stage_span over a row of 16-bit elements (type 1: bf16, 2: fp16), widened
// to float; type 0 is stage_span itself.
template <int NT = kThreads>
__device__ __forceinline__ void stage_span_any(float* dst, const void* src, int64_t base, int64_t n, int type) {
  if (type == 0) {
    stage_span<NT>(dst, static_cast<const float*>(src), base, n);
    return;
  }
  constexpr int kPer = kChunk;
  const unsigned short* s = static_cast<const unsigned short*>(src);
  unsigned short v[kPer];
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int64_t g = base + threadIdx.x + k * NT;
    v[k] = (g >= 0 && g < n) ? __ldg(s + g) : (unsigned short)0;
  }
#pragma unroll
  for (int k = 0; k < kPer; ++k)
    dst[threadIdx.x + k * NT] =
        type == 1 ? __uint_as_float((unsigned)v[k] << 16) : __half2float(__ushort_as_half(v[k]));
}

// dst[k * pitch + t] = src[k * src_pitch + t] for k < rows, t < cnt, by a CTA
// of kBlock threads with 8 loads per thread in flight at a time (one memory
// round trip for up to 8 * kBlock elements).  src must be read-only for the
// whole kernel.
template <int kBlock>
__device__ __forceinline__ void stage_rows(float* dst, int pitch, const float* src, int64_t src_pitch, int rows,
                                           int cnt) {
  const int n = rows * cnt;
  for (int base = threadIdx.x; base < n; base += 8 * kBlock) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * kBlock;
      const int k = i / max(cnt, 1), t = i - k * cnt;
      v[j] = i < n ? __ldg(src + k * src_pitch + t) : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = base + j * kBlock;
      const int k = i / max(cnt, 1), t = i - k * cnt;
      if (i < n) dst[k * pitch + t] = v[j];
    }
  }
}

// 4-byte asynchronous copy global -> shared; complete after cp_async_wait_all
// (then __syncthreads before other threads read the data)
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
// 16-byte asynchronous copy global -> shared (both addresses 16-byte aligned)
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src)
               : "memory");
}
// 4-byte asynchronous copy global -> shared that writes zero (and reads
// nothing) when `valid` is false; `src` must still be a valid address.
__device__ __forceinline__ void cp_async4_zfill(float* dst, const float* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }
// wait until at most N of this thread's committed groups are still in flight
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Asynchronous form of stage_rows: every thread only issues cp.async copies,
// so any number of stagings can be in flight together; the data is in place
// after cp_async_wait_all() and a CTA barrier.
template <int kBlock>
__device__ __forceinline__ void stage_rows_async(float* dst, int pitch, const float* src, int64_t src_pitch,
                                                 int rows, int cnt) {
  for (int k = 0; k < rows; ++k)
    for (int t = threadIdx.x; t < cnt; t += kBlock) cp_async4(dst + k * pitch + t, src + k * src_pitch + t);
}

// Asynchronous copy of `bytes` (a multiple of 16, both addresses 16-byte
// aligned) by a CTA of kBlock threads; complete as for stage_rows_async.
template <int kBlock>
__device__ __forceinline__ void copy_async(void* dst, const void* src, int bytes) {
  char* d = static_cast<char*>(dst);
  const char* s = static_cast<const char*>(src);
  for (int i = threadIdx.x; i < bytes / 16; i += kBlock) cp_async16(d + 16 * i, s + 16 * i);
}

// ---------------------------------------------------------------------------
// bulk copy (TMA, no multicast) shared -> global
// ---------------------------------------------------------------------------

// Makes this thread's earlier generic-proxy writes to shared memory visible
// to the async proxy (bulk copies); followed by a CTA barrier before the copy.
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from
// shared to global memory, tracked by the issuing thread's bulk async-group.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"((uint32_t)__cvta_generic_to_shared(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// the issuing thread's bulk copies have completed (their writes are done)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// bulk copy (TMA, no multicast) global -> shared, completed on an mbarrier
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// One thread initialises the barrier (one arrival per phase); a CTA barrier
// must follow before other threads wait on it.
__device__ __forceinline__ void mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(bar)) : "memory");
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// The issuing thread's arrival, announcing `bytes` of bulk copies that
// complete the current phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Copy of `bytes` (a multiple of 16, both addresses 16-byte aligned) from this
// GPU's global memory into this CTA's shared memory, signalled on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Tries (each a hardware-bounded suspend) before a wait on a bulk copy gives
// up; a copy of this GPU's memory lands within microseconds.
constexpr uint32_t kMbarTries = 1u << 16;

// Waits for phase `parity` of `bar` with a bounded number of tries; false if
// it did not complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMbarTries; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

// Device-side error flags, OR-ed into the plan's error word, which the host
// reads back (and clears) with pesq_plan_check.
enum : uint32_t {
  kErrBulkTimeout = 1u << 0,  // a bulk copy into shared memory did not complete in time
  kErrBadGeometry = 1u << 1,
};

}  // namespace pesq
