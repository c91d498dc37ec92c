// Shared device helpers for the sm_100a INT4 paged KV-cache kernels.
//
// Everything here is a thin wrapper over a single PTX instruction (mbarrier,
// TMA bulk / tensor copies, ldmatrix, movmatrix, mma.sync, lop3) so the
// kernels read as data flow.  No CUDA math-library code is reproduced.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/iris_b200.h"

#define IRIS_DEV __device__ __forceinline__

namespace iris {

// Bounded waits.  Each poll is an mbarrier.try_wait with a suspend-time
// hint, so a waiting warp sleeps in hardware (no issue slots burnt) until the
// phase completes or the hint expires.  A wait gives up after kWaitLimitNs of
// %globaltimer time (whatever the hardware does with the hint), records
// IRIS_ERR_PIPELINE_TIMEOUT and returns instead of hanging the GPU.
constexpr uint32_t kSuspendHintNs = 100000;        // 0.1 ms per poll at most
constexpr uint64_t kWaitLimitNs = 2000000000ull;   // 2 s per wait

IRIS_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

IRIS_DEV void set_error(int32_t* err, int32_t bits) {
  if (err != nullptr) atomicOr(err, bits);
}

IRIS_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
IRIS_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

IRIS_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

IRIS_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

IRIS_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

IRIS_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Returns false (and records the timeout) if the phase never completes.
IRIS_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int32_t* err, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) break;
  }
  set_error(err, IRIS_ERR_PIPELINE_TIMEOUT);
  return false;
}

IRIS_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int32_t* err) {
  return mbar_wait_bounded(smem_u32(bar), parity, err);
}

IRIS_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

IRIS_DEV uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

IRIS_DEV uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

IRIS_DEV void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// --------------------------------------------------------------- TMA copies
// 1-D bulk copy global -> shared, completion signalled on `bar` (tx bytes).
// Both addresses 16-byte aligned, bytes a multiple of 16.
IRIS_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 3-D tiled tensor copy global -> shared (no multicast).  c0 is the innermost
// coordinate; it is always 0 here (whole rows), so the 16-byte rule holds.
IRIS_DEV void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled tensor copy global -> shared (no multicast); c0 is always 0.
IRIS_DEV void tma_load_4d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// 5-D tiled tensor copy global -> shared (no multicast); c0 is always 0.
IRIS_DEV void tma_load_5d(void* dst, const CUtensorMap* map, int c0, int c1, int c2, int c3, int c4, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(smem_u32(bar))
      : "memory");
}

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) accesses of the same bytes.
IRIS_DEV void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bulk prefetch of a global range into L2 (16-byte aligned, size a multiple of 16).
IRIS_DEV void prefetch_l2_bulk(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}

IRIS_DEV void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------- programmatic dependent launch
// A kernel launched with programmatic stream serialization may start while
// the previous kernel of the stream is still running (once every CTA of that
// kernel has called grid_dependents_launch, or exited); grid_dependency_wait
// then blocks until the previous kernel has finished and its memory writes
// are visible.  Without the launch attribute both are no-ops.
IRIS_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
IRIS_DEV void grid_dependents_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------- warp-level matrix
IRIS_DEV void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

IRIS_DEV void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

IRIS_DEV uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// D = A * B + C, m16n8k16, fp16 inputs, fp32 accumulate.
IRIS_DEV void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

template <int kLut>
IRIS_DEV uint32_t lop3(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("lop3.b32 %0, %1, %2, %3, %4;" : "=r"(d) : "r"(a), "r"(b), "r"(c), "n"(kLut));
  return d;
}

IRIS_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// INT4 -> fp16 "magic number" conversion (the exponent-bias trick of
// Kim et al., "Who Says Elephants Can't Run?", 2022), with the two's-
// complement -> offset-binary flip folded into the same LOP3.
//
// lop3 truth table f(w, A, B): A=0,B=0 -> 0; A=0,B=1 -> 1; A=1,B=0 -> w;
// A=1,B=1 -> ~w.  With A selecting a nibble's bits and B holding 0x6400 plus
// the nibble's top bit, each fp16 half becomes 0x6400 | (n ^ 8) << shift,
// i.e. 1024 + (n + 8) for the low nibble of a byte and 1024 + 16 (n + 8) for
// the high nibble.  LUT = (~A & B) | (A & (w ^ B)) = 0x6A.
constexpr int kLutMagic = 0x6A;
IRIS_DEV uint32_t int4_lo_biased(uint32_t w) {  // halves: n + 1032 (nibbles 0 and 4)
  return lop3<kLutMagic>(w, 0x000f000fu, 0x64086408u);
}
IRIS_DEV uint32_t int4_hi_biased(uint32_t w) {  // halves: 16 n + 1152 (nibbles 1 and 5)
  return lop3<kLutMagic>(w, 0x00f000f0u, 0x64806480u);
}

IRIS_DEV uint32_t h2_as_u32(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
IRIS_DEV __half2 u32_as_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// Exact n from the biased forms above.
IRIS_DEV uint32_t int4_lo_exact(uint32_t w) {
  return h2_as_u32(__hsub2(u32_as_h2(int4_lo_biased(w)), __float2half2_rn(1032.0f)));
}
IRIS_DEV uint32_t int4_hi_exact(uint32_t w) {
  return h2_as_u32(__hfma2(u32_as_h2(int4_hi_biased(w)), __float2half2_rn(0.0625f), __float2half2_rn(-72.0f)));
}

IRIS_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

IRIS_DEV float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Host side: remember the last CUDA error of an entry point (per thread).
const char* record_cuda_error(cudaError_t e, const char* where);
cudaError_t clear_stale_cuda_error();

}  // namespace iris
