// L2 prefetch of weight ranges: the next op's packed weights are pulled from HBM into the 126 MB L2 while the
// current op computes, so the dependent chain of decode GEMVs reads its weights from L2 and HBM streams without the
// gaps between launches.
//
// One launch takes up to kMaxRanges byte ranges.  Each warp issues `cp.async.bulk.prefetch.L2` for chunks of
// kChunk bytes (16-byte aligned starts and sizes; the unaligned head and tail of a range go through per-line
// `prefetch.global.L2`).  The prefetches are fire-and-forget: the kernel retires as soon as they are issued, and the
// memory system fills L2 behind it.  The kernel is a programmatic-dependent launch that releases its successor at
// once and waits for its predecessor before it exits, so in a stream it neither delays the next op nor lets a later
// op see the stream's earlier work unfinished.
#include <cstring>

#include "fp4x_common.cuh"
#include "fp4x_host.h"

namespace fp4x {

namespace {

constexpr int kMaxRanges = 16;
constexpr int64_t kChunk = 32768;
constexpr int kPfThreads = 128;

struct PrefetchList {
  const uint8_t* ptr[kMaxRanges];
  int64_t bytes[kMaxRanges];
  int64_t chunk0[kMaxRanges + 1];  // prefix sums of the chunks per range
  int n;
};

FP4X_DEV void prefetch_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
FP4X_DEV void prefetch_line(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p) : "memory"); }

__global__ void __launch_bounds__(kPfThreads) prefetch_l2_kernel(const __grid_constant__ PrefetchList L) {
  pdl_launch_dependents();
  const int64_t total = L.chunk0[L.n];
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < total; c += stride) {
    int r = 0;
    while (r + 1 < L.n && L.chunk0[r + 1] <= c) ++r;
    const uint8_t* p = L.ptr[r];
    const int64_t n = L.bytes[r];
    const uint8_t* a = reinterpret_cast<const uint8_t*>(((uintptr_t)p + 15) & ~(uintptr_t)15);  // aligned start
    const int64_t head = a - p;
    const int64_t body = n > head ? (n - head) & ~(int64_t)15 : 0;
    const int64_t i = c - L.chunk0[r];
    const int64_t off = i * kChunk;
    if (off < body) {
      const int64_t len = body - off < kChunk ? body - off : kChunk;
      prefetch_bulk(a + off, (uint32_t)len);
    }
    if (i == 0) {  // the ragged head and tail, one 128-byte line at a time (at most two lines each)
      if (head > 0) prefetch_line(p);
      const int64_t tail = (n > head ? head + body : n);
      for (int64_t t = tail; t < n; t += 128) prefetch_line(p + t);
    }
  }
  // completion of this grid implies completion of the stream's previous work
  pdl_wait();
}

}  // namespace

}  // namespace fp4x

using namespace fp4x;

extern "C" {

int fp4x_prefetch_l2(const void* const* ptrs, const int64_t* bytes, int n, void* stream) {
  if (n < 0 || n > kMaxRanges || (n > 0 && (!ptrs || !bytes)))
    return fail(FP4X_ERR_INVALID_ARG, "prefetch takes 0.." + std::to_string(kMaxRanges) + " ranges");
  PrefetchList L;
  std::memset(&L, 0, sizeof(L));
  int k = 0;
  for (int i = 0; i < n; ++i) {
    if (bytes[i] < 0) return fail(FP4X_ERR_INVALID_ARG, "negative range size");
    if (bytes[i] == 0) continue;
    if (!ptrs[i]) return fail(FP4X_ERR_INVALID_ARG, "null range");
    L.ptr[k] = (const uint8_t*)ptrs[i];
    L.bytes[k] = bytes[i];
    L.chunk0[k + 1] = L.chunk0[k] + (bytes[i] + kChunk - 1) / kChunk;
    ++k;
  }
  L.n = k;
  if (k == 0) return FP4X_OK;
  const int64_t chunks = L.chunk0[k];
  int grid = (int)((chunks + kPfThreads - 1) / kPfThreads);
  if (grid > device_facts().sms) grid = device_facts().sms;
  return check_launch(launch_pdl(prefetch_l2_kernel, dim3(grid), dim3(kPfThreads), 0, (cudaStream_t)stream, L),
                      "prefetch_l2");
}

}  // extern "C"
