// LM-head kernels: exact top-C selection over coarse logits, exact MXFP8 / NVFP4 rescoring of the candidates,
// argmax, the fused fast / draft heads and the merge of per-shard candidates of a vocab-sharded head.
//
// Top-C order is total: value descending, then vocab index ascending (ties broken towards the smaller index).
// Selection = radix select on the order-preserving 32-bit key of each fp32 value:
//   1. topk_hist:   12-bit histogram of every row (smem per CTA, flushed with global atomics);
//   2. topk_filter: every CTA finds the bin that holds rank C and appends (key, index) of all values at or
//                   above that bin to a per-row candidate list;
//   3. topk_select: one CTA per row resolves the exact set inside the candidate list (three more radix digits,
//                   then index order among equal keys), marks it in a shared bitmap over the vocabulary and emits
//                   the indices in ascending order (deterministic, independent of the append order).  It then
//                   re-zeroes the histogram and the counter of its row, so the scratch is clean for the next call.
// If a candidate list overflows its capacity (pathological ties), the select CTA scans the whole row instead.
#include <algorithm>
#include <string>

#include "fp4x_common.cuh"
#include "fp4x_gemv.cuh"
#include "fp4x_host.h"

namespace fp4x {

constexpr int kHistBits = 12;
constexpr int kHistBins = 1 << kHistBits;
constexpr int kCandCap = 12288;         // candidate list capacity per row
constexpr int kMaxVocab = 262144;       // bitmap limit of the select kernel
constexpr int kSelThreads = 1024;

FP4X_DEV uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u ^ 0x80000000u);
}
FP4X_DEV float key_to_float(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k ^ 0x80000000u) : ~k;
  return __uint_as_float(u);
}

// ------------------------------------------------------------------------------------------------------
// 1. histogram
// ------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) topk_hist_kernel(const float* vals, int64_t ld, int V, int* hist) {
  __shared__ int h[kHistBins];
  const int m = blockIdx.y;
  for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) h[i] = 0;
  pdl_wait();
  __syncthreads();
  const int64_t per = ((int64_t)V + gridDim.x - 1) / gridDim.x;
  const int64_t b = per * blockIdx.x, e = min((int64_t)V, b + per);
  const float* row = vals + (int64_t)m * ld;
  for (int64_t i = b + threadIdx.x; i < e; i += blockDim.x) atomicAdd(&h[fkey(row[i]) >> (32 - kHistBits)], 1);
  __syncthreads();
  pdl_launch_dependents();
  int* gh = hist + (int64_t)m * kHistBins;
  for (int i = threadIdx.x; i < kHistBins; i += blockDim.x)
    if (h[i]) atomicAdd(&gh[i], h[i]);
}

// block-wide: the histogram bin (scanned from the top) that contains rank `need` (1-based); also returns the count
// strictly above that bin.  `h` is in shared memory, nb bins; all threads get the result.
// Exclusive prefix sum of one value per thread over the block (blockDim.x a multiple of 32, at most 1024), in
// thread order; wtot is shared scratch of 32 ints.  Every thread of the block must call it.
FP4X_DEV int block_exclusive_scan(int v, int* wtot) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) wtot[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int t = lane < nw ? wtot[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) ti += y;
    }
    wtot[lane] = ti - t;
  }
  __syncthreads();
  const int res = wtot[w] + incl - v;
  __syncthreads();
  return res;
}

template <int NT>
FP4X_DEV void find_rank_bin(const int* h, int nb, int need, int& bin_out, int& above_out, int* scratch) {
  // scratch: NT + 34 ints
  const int per = (nb + NT - 1) / NT;
  const int t = threadIdx.x;
  // thread t owns bins counted from the top: top index = nb-1 - (t*per + j)
  int tot = 0;
  for (int j = 0; j < per; ++j) {
    const int bi = nb - 1 - (t * per + j);
    if (bi >= 0) tot += h[bi];
  }
  const int before = block_exclusive_scan(tot, scratch + NT + 2);
  if (before < need && before + tot >= need) {
    int cum = before;
    for (int j = 0; j < per; ++j) {
      const int bi = nb - 1 - (t * per + j);
      if (bi < 0) break;
      if (cum + h[bi] >= need) {
        scratch[NT] = bi;
        scratch[NT + 1] = cum;
        break;
      }
      cum += h[bi];
    }
  }
  __syncthreads();
  bin_out = scratch[NT];
  above_out = scratch[NT + 1];
  __syncthreads();
}

// ------------------------------------------------------------------------------------------------------
// 2. filter: append (key, index) of every value in a bin >= the rank-C bin
// ------------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(512) topk_filter_kernel(const float* vals, int64_t ld, int V, int C,
                                                          const int* hist, int* cnt, uint64_t* cand) {
  __shared__ int h[kHistBins];
  __shared__ int scr[512 + 34];
  const int m = blockIdx.y;
  pdl_wait();
  for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) h[i] = hist[(int64_t)m * kHistBins + i];
  __syncthreads();
  int bstar, above;
  find_rank_bin<512>(h, kHistBins, C, bstar, above, scr);
  pdl_launch_dependents();
  const int64_t per = ((int64_t)V + gridDim.x - 1) / gridDim.x;
  const int64_t b = per * blockIdx.x, e = min((int64_t)V, b + per);
  const float* row = vals + (int64_t)m * ld;
  const int lane = threadIdx.x & 31;
  uint64_t* out = cand + (int64_t)m * kCandCap;
  for (int64_t base = b; base < e; base += blockDim.x) {
    const int64_t i = base + threadIdx.x;
    uint32_t key = 0;
    bool take = false;
    if (i < e) {
      key = fkey(row[i]);
      take = (int)(key >> (32 - kHistBits)) >= bstar;
    }
    const uint32_t mask = __ballot_sync(0xffffffffu, take);
    if (mask) {
      int pos0 = 0;
      const int leader = __ffs(mask) - 1;
      if (lane == leader) pos0 = atomicAdd(cnt + m, __popc(mask));
      pos0 = __shfl_sync(0xffffffffu, pos0, leader);
      if (take) {
        const int pos = pos0 + __popc(mask & ((1u << lane) - 1));
        if (pos < kCandCap) out[pos] = ((uint64_t)key << 32) | (uint32_t)i;
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------------
// 3. per-row exact selection
// ------------------------------------------------------------------------------------------------------
struct SelectShared {
  uint32_t sel[kMaxVocab / 32];   // selected indices
  uint32_t eq[kMaxVocab / 32];    // candidates whose key equals the final prefix
  int h[kHistBins];
  int scr[kSelThreads + 34];
  int wpre[kSelThreads + 1];
  int wtot[32];
};
// the candidate list (uint64) follows SelectShared in dynamic shared memory at a 16-byte aligned offset
constexpr size_t kListOffset = (sizeof(SelectShared) + 15) / 16 * 16;
static_assert(kListOffset % 16 == 0, "candidate list alignment");

// Candidate sources: the shared copy of the candidate list, or the whole row (overflow).
struct ListSrc {
  const uint64_t* c;
  int n;
  template <class F>
  FP4X_DEV void each(F f) const {
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const uint64_t v = c[i];
      f((uint32_t)(v >> 32), (uint32_t)v);
    }
  }
};
struct RowSrc {
  const float* row;
  int V;
  template <class F>
  FP4X_DEV void each(F f) const {
    for (int i = threadIdx.x; i < V; i += blockDim.x) f(fkey(row[i]), (uint32_t)i);
  }
};

// Marks the C best (key desc, index asc) of the source in S.sel.  Requires C <= number of candidates.
template <class Src>
FP4X_DEV void select_top(const Src& src, int C, int V, SelectShared& S) {
  const int nw = (V + 31) / 32;
  for (int i = threadIdx.x; i < nw; i += blockDim.x) {
    S.sel[i] = 0;
    S.eq[i] = 0;
  }
  int need = C;
  uint32_t prefix = 0;
  int pbits = 0;
  const int digits[3] = {12, 12, 8};
  bool done = false;
  for (int d = 0; d < 3 && !done; ++d) {
    const int bits = digits[d];
    const int shift = 32 - pbits - bits;
    const int nb = 1 << bits;
    for (int i = threadIdx.x; i < nb; i += blockDim.x) S.h[i] = 0;
    __syncthreads();
    const uint32_t pmask = pbits ? (0xffffffffu << (32 - pbits)) : 0u;
    src.each([&](uint32_t key, uint32_t idx) {
      if ((key & pmask) == prefix) atomicAdd(&S.h[(key >> shift) & (nb - 1)], 1);
    });
    __syncthreads();
    int bin, above;
    find_rank_bin<kSelThreads>(S.h, nb, need, bin, above, S.scr);
    const int inbin = S.h[bin];
    const bool all_fit = (need - above == inbin);
    src.each([&](uint32_t key, uint32_t idx) {
      if ((key & pmask) == prefix) {
        const int dg = (int)((key >> shift) & (nb - 1));
        if (dg > bin || (all_fit && dg == bin)) atomicOr(&S.sel[idx >> 5], 1u << (idx & 31));
      }
    });
    need -= above;
    prefix |= (uint32_t)bin << shift;
    pbits += bits;
    if (all_fit) done = true;
    __syncthreads();
  }
  if (!done && need > 0) {
    // equal keys: take the `need` smallest indices among the candidates equal to the full prefix
    src.each([&](uint32_t key, uint32_t idx) {
      if (key == prefix) atomicOr(&S.eq[idx >> 5], 1u << (idx & 31));
    });
    __syncthreads();
    // ordered prefix over eq words: per-thread contiguous word ranges
    const int per = (nw + blockDim.x - 1) / blockDim.x;
    const int w0 = threadIdx.x * per;
    int cnt = 0;
    for (int w = w0; w < min(nw, w0 + per); ++w) cnt += __popc(S.eq[w]);
    int before = block_exclusive_scan(cnt, S.wtot);
    for (int w = w0; w < min(nw, w0 + per) && before < need; ++w) {
      uint32_t bitsw = S.eq[w];
      while (bitsw && before < need) {
        const int bpos = __ffs(bitsw) - 1;
        bitsw &= bitsw - 1;
        atomicOr(&S.sel[w], 1u << bpos);
        ++before;
      }
    }
  }
  __syncthreads();
}

// Writes the selected indices of S.sel in ascending order (and the key-decoded value when `vals` is given).
FP4X_DEV void emit_selected(const SelectShared& S, int V, int C, int32_t* idx_out, float* val_out, const float* row) {
  const int nw = (V + 31) / 32;
  const int per = (nw + blockDim.x - 1) / blockDim.x;
  const int w0 = threadIdx.x * per;
  int cnt = 0;
  for (int w = w0; w < min(nw, w0 + per); ++w) cnt += __popc(S.sel[w]);
  int pos = block_exclusive_scan(cnt, const_cast<int*>(S.wtot));
  for (int w = w0; w < min(nw, w0 + per); ++w) {
    uint32_t b = S.sel[w];
    while (b) {
      const int bp = __ffs(b) - 1;
      b &= b - 1;
      const int idx = w * 32 + bp;
      if (pos < C) {
        idx_out[pos] = idx;
        if (val_out) val_out[pos] = row[idx];
      }
      ++pos;
    }
  }
}

__global__ void __launch_bounds__(kSelThreads) topk_select_kernel(const float* vals, int64_t ld, int V, int C,
                                                                  int* hist, int* cnt, const uint64_t* cand,
                                                                  int32_t* idx_out, int64_t idx_ld,
                                                                  float* val_out, int64_t val_ld) {
  extern __shared__ __align__(16) uint8_t smem_sel[];
  SelectShared& S = *reinterpret_cast<SelectShared*>(smem_sel);
  uint64_t* list = reinterpret_cast<uint64_t*>(smem_sel + kListOffset);
  const int m = blockIdx.x;
  pdl_wait();
  const int n = cnt[m];
  const float* row = vals + (int64_t)m * ld;
  if (n <= kCandCap) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) list[i] = cand[(int64_t)m * kCandCap + i];
    __syncthreads();
    select_top(ListSrc{list, n}, C, V, S);
  } else {
    select_top(RowSrc{row, V}, C, V, S);
  }
  pdl_launch_dependents();
  emit_selected(S, V, C, idx_out + (int64_t)m * idx_ld, val_out ? val_out + (int64_t)m * val_ld : nullptr, row);
  // leave the scratch of this row clean for the next call
  for (int i = threadIdx.x; i < kHistBins; i += blockDim.x) hist[(int64_t)m * kHistBins + i] = 0;
  if (threadIdx.x == 0) cnt[m] = 0;
}

// ------------------------------------------------------------------------------------------------------
// rescoring: one warp per candidate, exact products, fp32 sums
// ------------------------------------------------------------------------------------------------------
FP4X_DEV int64_t load_idx(const void* idx, int idx64, int64_t off) {
  return idx64 ? reinterpret_cast<const int64_t*>(idx)[off] : (int64_t)reinterpret_cast<const int32_t*>(idx)[off];
}

// out[m, row] = cast(exact) (when out != null); exact_out[m, c] = exact (when != null)
__global__ void __launch_bounds__(256) refine_mx8_kernel(void* out, int64_t out_ld, int out_dtype, const __nv_bfloat16* x,
                                                         int64_t x_ld, const void* idx, int idx64, int64_t idx_ld,
                                                         const uint8_t* w, const uint8_t* s, int M, int C, int K,
                                                         float* exact_out, int64_t ex_ld) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M * C) return;
  const int m = warp / C, c = warp - m * C;
  const int64_t row = load_idx(idx, idx64, (int64_t)m * idx_ld + c);
  const uint8_t* wr = w + row * K;
  const uint8_t* sr = s + row * (K / 32);
  const __nv_bfloat16* xr = x + (int64_t)m * x_ld;
  float acc = 0.f;
  for (int ch = lane; ch < K / 16; ch += 32) {
    const uint4 cw = __ldg(reinterpret_cast<const uint4*>(wr) + ch);
    const float sc = e8m0_to_f32(__ldg(sr + (ch >> 1)));
    const uint4 x0 = __ldg(reinterpret_cast<const uint4*>(xr) + 2 * ch);
    const uint4 x1 = __ldg(reinterpret_cast<const uint4*>(xr) + 2 * ch + 1);
    const uint32_t wv[4] = {cw.x, cw.y, cw.z, cw.w};
    const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t h0 = e4m3x2_to_f16x2(wv[q]), h1 = e4m3x2_to_f16x2(wv[q] >> 16);
      const float w0 = f16_bits_to_f32(h0 & 0xffffu) * sc, w1 = f16_bits_to_f32(h0 >> 16) * sc;
      const float w2 = f16_bits_to_f32(h1 & 0xffffu) * sc, w3 = f16_bits_to_f32(h1 >> 16) * sc;
      acc = fmaf(w0, bf16_bits_to_f32(xv[2 * q] & 0xffffu), acc);
      acc = fmaf(w1, bf16_bits_to_f32(xv[2 * q] >> 16), acc);
      acc = fmaf(w2, bf16_bits_to_f32(xv[2 * q + 1] & 0xffffu), acc);
      acc = fmaf(w3, bf16_bits_to_f32(xv[2 * q + 1] >> 16), acc);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) {
    if (out) store_out(out, out_dtype, (int64_t)m * out_ld + row, acc);
    if (exact_out) exact_out[(int64_t)m * ex_ld + c] = acc;
  }
}

// out[m, c] = gs * sum_k bf16(e2m1 * e4m3 scale) * x (fp32)
__global__ void __launch_bounds__(256) refine_nv4_kernel(float* out, int64_t out_ld, const __nv_bfloat16* x,
                                                         int64_t x_ld, const void* idx, int idx64, int64_t idx_ld,
                                                         const uint8_t* wp, const uint8_t* s, float gs, int M, int C,
                                                         int K) {
  pdl_wait();
  pdl_launch_dependents();
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M * C) return;
  const int m = warp / C, c = warp - m * C;
  const int64_t row = load_idx(idx, idx64, (int64_t)m * idx_ld + c);
  const uint8_t* wr = wp + row * (K / 2);
  const uint8_t* sr = s + row * (K / 16);
  const __nv_bfloat16* xr = x + (int64_t)m * x_ld;
  float acc = 0.f;
  for (int ch = lane; ch < K / 32; ch += 32) {  // 16 bytes = 32 k = two scale groups
    const uint4 cw = __ldg(reinterpret_cast<const uint4*>(wr) + ch);
    const float s0 = e4m3_to_f32(__ldg(sr + 2 * ch)), s1 = e4m3_to_f32(__ldg(sr + 2 * ch + 1));
    const uint32_t wv[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 xq = __ldg(reinterpret_cast<const uint4*>(xr) + 4 * ch + q);
      const uint32_t xv[4] = {xq.x, xq.y, xq.z, xq.w};
      const float sc = q < 2 ? s0 : s1;
#pragma unroll
      for (int bb = 0; bb < 4; ++bb) {
        const uint32_t h = e2m1x2_to_f16x2(wv[q] >> (8 * bb));
        const float a = bf16_round(f16_bits_to_f32(h & 0xffffu) * sc);
        const float b = bf16_round(f16_bits_to_f32(h >> 16) * sc);
        acc = fmaf(a, bf16_bits_to_f32(xv[bb] & 0xffffu), acc);
        acc = fmaf(b, bf16_bits_to_f32(xv[bb] >> 16), acc);
      }
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) out[(int64_t)m * out_ld + c] = acc * gs;
}

// argmax over exact values with indices in ascending order: the first maximum wins (smallest index)
__global__ void argmax_kernel(const float* vals, int64_t ld, const int32_t* idx, int64_t idx_ld, int C,
                              int32_t* out) {
  pdl_wait();
  pdl_launch_dependents();
  const int m = blockIdx.x, lane = threadIdx.x;
  float best = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  for (int c = lane; c < C; c += 32) {
    const float v = vals[(int64_t)m * ld + c];
    const int id = idx[(int64_t)m * idx_ld + c];
    if (v > best || (v == best && id < bi) || (bi == 0x7fffffff && !(v == v))) {
      best = v;
      bi = id;
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) out[m] = bi;
}

// ------------------------------------------------------------------------------------------------------
// draft head output: -inf everywhere, exact values at ids[idx]
// ------------------------------------------------------------------------------------------------------
__global__ void fill_neg_inf_bf16(__nv_bfloat16* full, int64_t n) {
  pdl_wait();
  pdl_launch_dependents();
  const __nv_bfloat16 ninf = __ushort_as_bfloat16((unsigned short)0xFF80u);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    full[i] = ninf;
}

__global__ void draft_scatter_kernel(__nv_bfloat16* full, int64_t full_ld, const int64_t* ids, const int32_t* idx,
                                     const float* vals, int M, int C) {
  pdl_wait();
  pdl_launch_dependents();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= M * C) return;
  const int m = t / C;
  full[(int64_t)m * full_ld + ids[idx[t]]] = __float2bfloat16_rn(vals[t]);
}

// ------------------------------------------------------------------------------------------------------
// merge of per-shard candidates (vocab-sharded head): global top-C by coarse value, exact argmax
// ------------------------------------------------------------------------------------------------------
struct MergeSrc {
  const float* coarse;  // [P][M][C]
  const int32_t* gidx;
  int P, M, C, m;
  template <class F>
  FP4X_DEV void each(F f) const {
    for (int i = threadIdx.x; i < P * C; i += blockDim.x) {
      const int p = i / C, c = i - p * C;
      const int64_t off = ((int64_t)p * M + m) * C + c;
      f(fkey(coarse[off]), (uint32_t)gidx[off]);
    }
  }
};

__global__ void __launch_bounds__(kSelThreads) head_merge_kernel(const float* coarse, const float* exact,
                                                                 const int32_t* gidx, int P, int M, int C, int V,
                                                                 int32_t* idx_out, float* coarse_out,
                                                                 float* exact_out, int32_t* argmax_out) {
  extern __shared__ __align__(16) uint8_t smem_sel[];
  SelectShared& S = *reinterpret_cast<SelectShared*>(smem_sel);
  const int m = blockIdx.x;
  pdl_wait();
  MergeSrc src{coarse, gidx, P, M, C, m};
  select_top(src, C, V, S);
  // position of each selected global index = number of selected indices below it
  const int nw = (V + 31) / 32;
  const int per = (nw + blockDim.x - 1) / blockDim.x;
  const int w0 = threadIdx.x * per;
  int cnt = 0;
  for (int w = w0; w < min(nw, w0 + per); ++w) cnt += __popc(S.sel[w]);
  S.wpre[threadIdx.x] = block_exclusive_scan(cnt, S.wtot);
  __syncthreads();
  for (int i = threadIdx.x; i < P * C; i += blockDim.x) {
    const int p = i / C, c = i - p * C;
    const int64_t off = ((int64_t)p * M + m) * C + c;
    const uint32_t g = (uint32_t)gidx[off];
    const uint32_t word = S.sel[g >> 5];
    if (!((word >> (g & 31)) & 1u)) continue;
    // rank among selected: prefix of this thread-range word block + popcount of earlier words in its range
    const int w = g >> 5;
    const int owner = w / per;
    int pos = S.wpre[owner];
    for (int ww = owner * per; ww < w; ++ww) pos += __popc(S.sel[ww]);
    pos += __popc(word & ((1u << (g & 31)) - 1u));
    if (pos < C) {
      idx_out[(int64_t)m * C + pos] = (int32_t)g;
      if (coarse_out) coarse_out[(int64_t)m * C + pos] = coarse[off];
      exact_out[(int64_t)m * C + pos] = exact[off];
    }
  }
  __syncthreads();
  pdl_launch_dependents();
  if (threadIdx.x < 32) {
    float best = -__int_as_float(0x7f800000);
    int bi = 0x7fffffff;
    for (int c = threadIdx.x; c < C; c += 32) {
      const float v = exact_out[(int64_t)m * C + c];
      const int id = idx_out[(int64_t)m * C + c];
      if (v > best || (v == best && id < bi)) {
        best = v;
        bi = id;
      }
    }
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) argmax_out[m] = bi;
  }
}

// ------------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------------
static size_t select_smem() { return kListOffset + (size_t)kCandCap * sizeof(uint64_t); }
static size_t merge_smem() { return sizeof(SelectShared); }

struct TopkScratch {
  int* hist;        // counters: [M][4096]
  int* cnt;         // counters: [M]
  uint64_t* cand;   // workspace: [M][kCandCap]
};

static int64_t topk_counters(int64_t m) { return m * (kHistBins + 1); }
static size_t topk_ws(int64_t m) { return (size_t)m * kCandCap * sizeof(uint64_t); }

static int check_topk(int64_t m, int64_t v, int64_t c) {
  if (m < 1 || m > 64) return fail(FP4X_ERR_INVALID_ARG, "rows must be in 1..64");
  if (v < 1 || v > kMaxVocab) return fail(FP4X_ERR_UNSUPPORTED, "vocabulary per row must be <= 262144");
  if (c < 1 || c > v || c > 4096) return fail(FP4X_ERR_INVALID_ARG, "C must be in 1..min(V, 4096)");
  return FP4X_OK;
}

static int run_topk(const float* vals, int64_t ld, int64_t m, int64_t v, int64_t c, int32_t* idx, int64_t idx_ld,
                    float* val_out, int64_t val_ld, const TopkScratch& sc, cudaStream_t st) {
  int rc;
  const int sms = device_facts().sms;
  const int bx = (int)std::max<int64_t>(1, std::min<int64_t>((2 * sms + m - 1) / m, (v + 4095) / 4096));
  if ((rc = check_launch(launch_pdl(topk_hist_kernel, dim3(bx, (unsigned)m), dim3(512), 0, st, vals, ld, (int)v,
                                    sc.hist),
                         "topk hist")))
    return rc;
  if ((rc = check_launch(launch_pdl(topk_filter_kernel, dim3(bx, (unsigned)m), dim3(512), 0, st, vals, ld, (int)v,
                                    (int)c, (const int*)sc.hist, sc.cnt, sc.cand),
                         "topk filter")))
    return rc;
  const int smem = (int)select_smem();
  cudaError_t e = ensure_smem_attr((const void*)topk_select_kernel, smem);
  if (e != cudaSuccess) return check_launch(e, "topk select attr");
  return check_launch(launch_pdl(topk_select_kernel, dim3((unsigned)m), dim3(kSelThreads), smem, st, vals, ld, (int)v,
                                 (int)c, sc.hist, sc.cnt, (const uint64_t*)sc.cand, idx, idx_ld, val_out, val_ld),
                      "topk select");
}

static int launch_refine_mx8(void* out, int64_t out_ld, int out_dtype, const void* x, int64_t x_ld, const void* idx,
                             int idx64, int64_t idx_ld, const void* w, const void* s, int64_t m, int64_t c, int64_t k,
                             float* exact, int64_t ex_ld, cudaStream_t st) {
  const int64_t warps = m * c;
  return check_launch(launch_pdl(refine_mx8_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, st, out, out_ld,
                                 out_dtype, (const __nv_bfloat16*)x, x_ld, idx, idx64, idx_ld, (const uint8_t*)w,
                                 (const uint8_t*)s, (int)m, (int)c, (int)k, exact, ex_ld),
                      "refine mx8");
}

static int launch_refine_nv4(float* out, int64_t out_ld, const void* x, int64_t x_ld, const void* idx, int idx64,
                             int64_t idx_ld, const void* wp, const void* s, float gs, int64_t m, int64_t c, int64_t k,
                             cudaStream_t st) {
  const int64_t warps = m * c;
  return check_launch(launch_pdl(refine_nv4_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, st, out, out_ld,
                                 (const __nv_bfloat16*)x, x_ld, idx, idx64, idx_ld, (const uint8_t*)wp,
                                 (const uint8_t*)s, gs, (int)m, (int)c, (int)k),
                      "refine nv4");
}

// scratch layout of the fused heads: workspace = [coarse fp32 M*V][exact fp32 M*C][idx int32 M*C]
//                                               [gemv ws][topk cand]; counters = [gemv][topk hist+cnt]
struct HeadLayout {
  size_t off_coarse, off_exact, off_idx, off_gemv, off_cand, ws_bytes;
  int64_t cnt_gemv, cnt_topk;
  size_t gemv_ws;
};

static size_t al256(size_t v) { return (v + 255) / 256 * 256; }

static int head_layout(int64_t m, int64_t V, int64_t K, int64_t C, int group, HeadLayout& L) {
  size_t gws = 0;
  int64_t gcnt = 0;
  int rc = fp4x_gemv_query(FP4X_FMT_INT2, m, V, K, 1, group, &gws, &gcnt);
  if (rc) return rc;
  L.off_coarse = 0;
  L.off_exact = al256((size_t)m * V * 4);
  L.off_idx = L.off_exact + al256((size_t)m * C * 4);
  L.off_gemv = L.off_idx + al256((size_t)m * C * 4);
  L.off_cand = L.off_gemv + al256(gws);
  L.ws_bytes = L.off_cand + al256(topk_ws(m));
  L.gemv_ws = gws;
  L.cnt_gemv = gcnt;
  L.cnt_topk = topk_counters(m);
  return FP4X_OK;
}

}  // namespace fp4x

using namespace fp4x;

extern "C" {

int fp4x_topk_query(int64_t m, int64_t v, int64_t c, size_t* ws_bytes, int64_t* n_counters) {
  int rc = check_topk(m, v, c);
  if (rc) return rc;
  if (ws_bytes) *ws_bytes = topk_ws(m);
  if (n_counters) *n_counters = topk_counters(m);
  return FP4X_OK;
}

int fp4x_topk(const float* vals, int64_t ld, int64_t m, int64_t v, int64_t c, int32_t* idx_out, int64_t idx_ld,
              float* val_out, int64_t val_ld, void* ws, size_t ws_bytes, int32_t* counters, int64_t n_counters,
              void* stream) {
  int rc = check_topk(m, v, c);
  if (rc) return rc;
  if (!vals || !idx_out) return fail(FP4X_ERR_INVALID_ARG, "null pointer");
  if (!ws || ws_bytes < topk_ws(m) || !counters || n_counters < topk_counters(m))
    return fail(FP4X_ERR_WORKSPACE, "scratch too small (see fp4x_topk_query)");
  TopkScratch sc{counters, counters + m * kHistBins, (uint64_t*)ws};
  return run_topk(vals, ld, m, v, c, idx_out, idx_ld, val_out, val_ld, sc, (cudaStream_t)stream);
}

int fp4x_refine_mx8(void* out, int64_t out_ld, int out_dtype, const void* x, int64_t x_ld, const void* idx, int idx64,
                    int64_t idx_ld, const void* w, const void* s, int64_t m, int64_t c, int64_t k, float* exact_out,
                    int64_t exact_ld, void* stream) {
  if (!x || !idx || !w || !s || (!out && !exact_out)) return fail(FP4X_ERR_INVALID_ARG, "null pointer");
  if (m < 1 || c < 1 || k % 32 || !aligned(x, 16) || x_ld % 8 || !aligned(w, 16) || k % 16)
    return fail(FP4X_ERR_UNSUPPORTED, "refine_mx8 needs K % 32 == 0 and 16-byte aligned rows");
  if (out_dtype < 0 || out_dtype > 2) return fail(FP4X_ERR_INVALID_ARG, "bad out_dtype");
  return launch_refine_mx8(out, out_ld, out_dtype, x, x_ld, idx, idx64, idx_ld, w, s, m, c, k, exact_out, exact_ld,
                           (cudaStream_t)stream);
}

int fp4x_refine_nv4(float* out, int64_t out_ld, const void* x, int64_t x_ld, const void* idx, int idx64, int64_t idx_ld,
                    const void* wp, const void* s, float gs, int64_t m, int64_t c, int64_t k, void* stream) {
  if (!out || !x || !idx || !wp || !s) return fail(FP4X_ERR_INVALID_ARG, "null pointer");
  if (m < 1 || c < 1 || k % 32 || !aligned(x, 16) || x_ld % 8 || !aligned(wp, 16))
    return fail(FP4X_ERR_UNSUPPORTED, "refine_nv4 needs K % 32 == 0 and 16-byte aligned rows");
  return launch_refine_nv4(out, out_ld, x, x_ld, idx, idx64, idx_ld, wp, s, gs, m, c, k, (cudaStream_t)stream);
}

int fp4x_argmax_candidates(const float* vals, int64_t ld, const int32_t* idx, int64_t idx_ld, int64_t m, int64_t c,
                           int32_t* out, void* stream) {
  if (!vals || !idx || !out || m < 1 || c < 1) return fail(FP4X_ERR_INVALID_ARG, "bad argument");
  return check_launch(launch_pdl(argmax_kernel, dim3((unsigned)m), dim3(32), 0, (cudaStream_t)stream, vals, ld, idx,
                                 idx_ld, (int)c, out),
                      "argmax");
}

int fp4x_fast_head_query(int64_t m, int64_t v, int64_t k, int64_t c, int group, size_t* ws_bytes,
                         int64_t* n_counters) {
  int rc = check_topk(m, v, c);
  if (rc) return rc;
  if (m > 16) return fail(FP4X_ERR_INVALID_ARG, "M must be in 1..16");
  HeadLayout L;
  if ((rc = head_layout(m, v, k, c, group, L))) return rc;
  if (ws_bytes) *ws_bytes = L.ws_bytes;
  if (n_counters) *n_counters = L.cnt_gemv + L.cnt_topk;
  return FP4X_OK;
}

int fp4x_fast_head(const void* x, int64_t x_ld, const void* p, const void* s, int group, const void* w8,
                   const void* s8, int64_t m, int64_t v, int64_t k, int64_t c, void* full_bf16, int64_t full_ld,
                   int32_t* idx_out, float* exact_out, float* coarse_out, int32_t* argmax_out, void* ws,
                   size_t ws_bytes, int32_t* counters, int64_t n_counters, void* stream) {
  int rc = check_topk(m, v, c);
  if (rc) return rc;
  if (m > 16) return fail(FP4X_ERR_INVALID_ARG, "M must be in 1..16");
  HeadLayout L;
  if ((rc = head_layout(m, v, k, c, group, L))) return rc;
  if (!ws || ws_bytes < L.ws_bytes || !counters || n_counters < L.cnt_gemv + L.cnt_topk)
    return fail(FP4X_ERR_WORKSPACE, "scratch too small (see fp4x_fast_head_query)");
  if (!aligned(ws, 256)) return fail(FP4X_ERR_UNSUPPORTED, "workspace must be 256-byte aligned");
  if (full_bf16 && full_ld != v) return fail(FP4X_ERR_UNSUPPORTED, "full logits must be contiguous [M, V]");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* base = (uint8_t*)ws;
  float* coarse = (float*)(base + L.off_coarse);
  float* exact = exact_out ? exact_out : (float*)(base + L.off_exact);
  int32_t* idx = idx_out ? idx_out : (int32_t*)(base + L.off_idx);
  // 1. coarse INT2 logits (fp32 for ranking, bf16 copy into the full logits)
  if ((rc = fp4x_int2_logits(x, x_ld, p, s, group, coarse, v, FP4X_F32, full_bf16, m, v, k, base + L.off_gemv,
                             L.gemv_ws, counters, L.cnt_gemv, stream)))
    return rc;
  // 2. exact top-C of the fp32 coarse logits
  TopkScratch sc{counters + L.cnt_gemv, counters + L.cnt_gemv + m * kHistBins, (uint64_t*)(base + L.off_cand)};
  if ((rc = run_topk(coarse, v, m, v, c, idx, c, coarse_out, c, sc, st))) return rc;
  // 3. exact MXFP8 rescoring, scattered into the full logits
  if ((rc = launch_refine_mx8(full_bf16, full_ld, FP4X_BF16, x, x_ld, idx, 0, c, w8, s8, m, c, k, exact, c, st)))
    return rc;
  // 4. argmax of the exact values
  if (argmax_out)
    return check_launch(launch_pdl(argmax_kernel, dim3((unsigned)m), dim3(32), 0, st, (const float*)exact, c,
                                   (const int32_t*)idx, c, (int)c, argmax_out),
                        "argmax");
  return FP4X_OK;
}

int fp4x_draft_head(const void* x, int64_t x_ld, const void* p, const void* s, int group, const void* wp,
                    const void* sn, float gs, int64_t m, int64_t v, int64_t k, int64_t c, int32_t* idx_out,
                    float* vals_out, const int64_t* ids, void* full_bf16, int64_t full_ld, int64_t full_v, void* ws,
                    size_t ws_bytes, int32_t* counters, int64_t n_counters, void* stream) {
  int rc = check_topk(m, v, c);
  if (rc) return rc;
  if (m > 16) return fail(FP4X_ERR_INVALID_ARG, "M must be in 1..16");
  if (!idx_out || !vals_out) return fail(FP4X_ERR_INVALID_ARG, "null output");
  HeadLayout L;
  if ((rc = head_layout(m, v, k, c, group, L))) return rc;
  if (!ws || ws_bytes < L.ws_bytes || !counters || n_counters < L.cnt_gemv + L.cnt_topk)
    return fail(FP4X_ERR_WORKSPACE, "scratch too small (see fp4x_fast_head_query)");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* base = (uint8_t*)ws;
  float* coarse = (float*)(base + L.off_coarse);
  if ((rc = fp4x_int2_logits(x, x_ld, p, s, group, coarse, v, FP4X_F32, nullptr, m, v, k, base + L.off_gemv,
                             L.gemv_ws, counters, L.cnt_gemv, stream)))
    return rc;
  TopkScratch sc{counters + L.cnt_gemv, counters + L.cnt_gemv + m * kHistBins, (uint64_t*)(base + L.off_cand)};
  if ((rc = run_topk(coarse, v, m, v, c, idx_out, c, nullptr, 0, sc, st))) return rc;
  if ((rc = launch_refine_nv4(vals_out, c, x, x_ld, idx_out, 0, c, wp, sn, gs, m, c, k, st))) return rc;
  if (full_bf16 && ids) {
    const int64_t n = m * full_ld;
    if ((rc = check_launch(launch_pdl(fill_neg_inf_bf16, dim3(256), dim3(256), 0, st, (__nv_bfloat16*)full_bf16, n),
                           "fill")))
      return rc;
    (void)full_v;
    return check_launch(launch_pdl(draft_scatter_kernel, dim3((unsigned)((m * c + 255) / 256)), dim3(256), 0, st,
                                   (__nv_bfloat16*)full_bf16, full_ld, ids, (const int32_t*)idx_out,
                                   (const float*)vals_out, (int)m, (int)c),
                        "draft scatter");
  }
  return FP4X_OK;
}

int fp4x_head_merge(const float* coarse, const float* exact, const int32_t* gidx, int64_t parts, int64_t m, int64_t c,
                    int64_t v, int32_t* idx_out, float* coarse_out, float* exact_out, int32_t* argmax_out,
                    void* stream) {
  if (!coarse || !exact || !gidx || !idx_out || !exact_out || !argmax_out) return fail(FP4X_ERR_INVALID_ARG, "null pointer");
  if (parts < 1 || parts > 64 || m < 1 || c < 1 || v < 1 || v > kMaxVocab)
    return fail(FP4X_ERR_INVALID_ARG, "bad merge shape");
  const int smem = (int)merge_smem();
  cudaError_t e = ensure_smem_attr((const void*)head_merge_kernel, smem);
  if (e != cudaSuccess) return check_launch(e, "merge attr");
  return check_launch(launch_pdl(head_merge_kernel, dim3((unsigned)m), dim3(kSelThreads), smem, (cudaStream_t)stream,
                                 coarse, exact, gidx, (int)parts, (int)m, (int)c, (int)v, idx_out, coarse_out,
                                 exact_out, argmax_out),
                      "head merge");
}

}  // extern "C"
