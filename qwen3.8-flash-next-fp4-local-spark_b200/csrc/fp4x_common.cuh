// Shared device helpers for the fp4x sm_100a kernels: bulk-copy / mbarrier plumbing with bounded waits,
// programmatic-dependent-launch controls, exact low-precision conversions and the warp-level MMA.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#define FP4X_DEV __device__ __forceinline__

namespace fp4x {

// ------------------------------------------------------------------------------------------------------
// error word: kernels never trap; a wait that gives up records a code here and the kernel returns.
// ------------------------------------------------------------------------------------------------------
enum DevError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,   // an mbarrier wait ran past its deadline
};

// the word lives in one translation unit; kernels receive its address as a parameter
FP4X_DEV void set_dev_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

FP4X_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Launch timeline, a diagnostic compiled only into libraries built with FP4X_TIMELINE (the stamp sites, even when
// not taken, cost the product kernels about 0.3 µs per launch): kTlWords globaltimer words per launch, recorded
// while the host has installed a buffer (fp4x_timeline_begin).  kTlStartFirst and kTlWaitFirst keep the earliest
// stamp of their event over the launch's CTAs (atomicMin; the host sets them to all ones), the others the latest
// (atomicMax; they start at zero).  FP4X_TL(statements) keeps a stamp site in the timeline build only.
enum TlWord {
  kTlStartFirst = 0,  // CTA start
  kTlStartLast,
  kTlWaitLast,        // return from the wait for the previous launch
  kTlXLanded,         // activation rows copied into shared memory
  kTlStaged,          // activations converted (and, NVFP4 on tensor cores, token maxima known)
  kTlFirstStage,      // first weight stage ready
  kTlLoopDone,        // accumulation done (consumer thread 0 / the MMA completion)
  kTlHandover,        // the two k-groups' partial sums combined
  kTlReduced,         // cross-CTA partial sums combined, epilogue starts
  kTlStored,          // outputs stored
  kTlWaitFirst,
  kTlWords = 16
};
#ifdef FP4X_TIMELINE
#define FP4X_TL(...) __VA_ARGS__
FP4X_DEV void tl_first(unsigned long long* tl, int i) {
  if (tl) atomicMin(tl + i, (unsigned long long)global_ns());
}
FP4X_DEV void tl_last(unsigned long long* tl, int i) {
  if (tl) atomicMax(tl + i, (unsigned long long)global_ns());
}
#else
#define FP4X_TL(...)
#endif

// ------------------------------------------------------------------------------------------------------
// programmatic dependent launch
// ------------------------------------------------------------------------------------------------------
FP4X_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FP4X_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------------------------------------------
// shared-memory addresses, mbarriers, bulk and async copies
// ------------------------------------------------------------------------------------------------------
FP4X_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

FP4X_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
FP4X_DEV void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

FP4X_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

FP4X_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
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

// Bounded wait: gives up after `limit_ns` of wall time, records kDevWaitTimeout and returns false.
FP4X_DEV bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int* err, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > limit_ns) {
      set_dev_error(err, kDevWaitTimeout);
      return false;
    }
  }
}

// ---- thread-block clusters (distributed shared memory) ----
FP4X_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// all threads of all CTAs of the cluster (the CTAs of a cluster are co-scheduled, so every CTA reaches it)
FP4X_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the shared::cluster address of `addr` (a shared::cta address of this CTA) in the CTA of rank `rank`
FP4X_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// asynchronous 16-byte store into another CTA of the cluster that completes its bytes on that CTA's mbarrier
// (complete_tx): the receiver's wait on the barrier makes the data visible, no release fence or arrival is needed
FP4X_DEV void st_async_v4(uint32_t cluster_addr, float a, float b, float c, float d, uint32_t cluster_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                   cluster_addr),
               "f"(a), "f"(b), "f"(c), "f"(d), "r"(cluster_bar)
               : "memory");
}
FP4X_DEV bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait whose completion acquires writes released at cluster scope by other CTAs
FP4X_DEV bool mbar_wait_bounded_cluster(uint32_t bar, uint32_t parity, int* err, uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 255u) == 0 && global_ns() - t0 > limit_ns) {
      set_dev_error(err, kDevWaitTimeout);
      return false;
    }
  }
}

// one contiguous global -> shared copy handled by the bulk-copy engine; completes on `bar` (tx bytes)
FP4X_DEV void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// 4-byte asynchronous copy (the scale rows, which need not be 16-byte aligned)
FP4X_DEV void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// arrive on `bar` once all of this thread's prior cp.async copies have landed (counts as one arrival)
FP4X_DEV void cp_async_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}
// order this thread's earlier generic-proxy shared accesses before later async-proxy (bulk copy) writes
FP4X_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

FP4X_DEV uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
FP4X_DEV uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
FP4X_DEV uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
FP4X_DEV uint32_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
FP4X_DEV uint32_t lds8(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
FP4X_DEV void sts64(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};" ::"r"(a), "r"(x), "r"(y) : "memory");
}
FP4X_DEV void sts16(uint32_t a, uint32_t x) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"((unsigned short)x) : "memory");
}

// ------------------------------------------------------------------------------------------------------
// byte permute and exact conversions
// ------------------------------------------------------------------------------------------------------
FP4X_DEV uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}

// two e4m3 bytes (low byte -> low half) to f16x2; exact for every e4m3 value
FP4X_DEV uint32_t e4m3x2_to_f16x2(uint32_t v16) {
  uint32_t d;
  uint16_t h = (uint16_t)v16;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(d) : "h"(h));
  return d;
}

// one byte holding two e2m1 nibbles (low nibble -> low half) to f16x2; exact
FP4X_DEV uint32_t e2m1x2_to_f16x2(uint32_t byte_in_low) {
  uint32_t d;
  uint16_t h = (uint16_t)(byte_in_low & 0xffu);
  asm("{\n\t.reg .b8 t;\n\tcvt.u8.u16 t, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(d) : "h"(h));
  return d;
}

FP4X_DEV uint32_t hadd2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
FP4X_DEV uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
FP4X_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
FP4X_DEV uint32_t pack_f16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}
// packed fp32 pairs (sm_100 f32x2 arithmetic; each lane rounds exactly like the scalar instruction)
FP4X_DEV uint64_t f32x2_from_bits(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
FP4X_DEV uint64_t f32x2_splat(float v) { return f32x2_from_bits(__float_as_uint(v), __float_as_uint(v)); }
FP4X_DEV uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
FP4X_DEV uint64_t f32x2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
FP4X_DEV uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
// the two fp32 lanes rounded to nearest-even bf16: low lane -> low half
FP4X_DEV uint32_t f32x2_to_bf16x2(uint64_t v) {
  uint32_t lo, hi, d;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "r"(hi), "r"(lo));
  return d;
}

FP4X_DEV float bf16_bits_to_f32(uint32_t b16) { return __uint_as_float(b16 << 16); }
FP4X_DEV float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
FP4X_DEV float f16_bits_to_f32(uint32_t h) { return __half2float(__ushort_as_half((unsigned short)h)); }

// e8m0 byte -> 2^(e-127) as fp32 (e = 0 gives the subnormal 2^-127, e = 255 gives inf as exp2(128) does)
FP4X_DEV float e8m0_to_f32(uint32_t e) { return __uint_as_float(e ? (e << 23) : 0x00400000u); }

// one e4m3 byte -> fp32 (exact)
FP4X_DEV float e4m3_to_f32(uint32_t b) {
  uint32_t h = e4m3x2_to_f16x2(b & 0xffu);
  return f16_bits_to_f32(h & 0xffffu);
}

// logistic function in fp32, the same expression for every kernel that needs it
FP4X_DEV float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// ------------------------------------------------------------------------------------------------------
// warp MMA m16n8k16, fp32 accumulate
// ------------------------------------------------------------------------------------------------------
FP4X_DEV void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}
FP4X_DEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, const float (&c)[4]) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

// ------------------------------------------------------------------------------------------------------
// output casts
// ------------------------------------------------------------------------------------------------------
enum OutDtype : int { kOutBF16 = 0, kOutF16 = 1, kOutF32 = 2 };

FP4X_DEV void store_out(void* out, int dtype, int64_t idx, float v) {
  if (dtype == kOutBF16)
    reinterpret_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else if (dtype == kOutF16)
    reinterpret_cast<__half*>(out)[idx] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(out)[idx] = v;
}

}  // namespace fp4x
