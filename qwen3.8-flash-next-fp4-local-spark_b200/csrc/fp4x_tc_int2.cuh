// INT2 coarse LM-head logits on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// out[m, n] = sum_k x[m, k] * bf16((code[n, k] - 1.5) * f32(s[n, k / g]))  -- the reference's _int2_head
// (x/fp4x_kernels.py:304-325, ROW_SCALE off) with g = 16 or 32 and fp16 scales.
//
// A 2-bit weight cannot be handed to a block-scaled MMA as stored: the reference rounds every (code - 1.5) * s to
// bf16, and neither e4m3 nor e8m0 block scales can carry an fp16 s.  So the weights are decoded, but straight into
// tensor memory: the MMA (kind::f16, bf16 x bf16 -> fp32) reads its A operand from tensor memory, so a decoded
// weight costs one register on its way from the 2-bit code to the tensor core and never touches shared memory.
//
//   decode: a 32-bit code word holds the 16 codes of one 16-k group (byte j: k = 4j + t at bit pair ORDER[t],
//   ORDER = 0, 2, 1, 3; x/fp4x_kernels.py:327-328).  The group's four bf16 values -1.5s, -0.5s, 0.5s, 1.5s are a
//   byte table (two registers), and one byte permute per two weights looks them up, selected by the codes of one bit
//   pair of two bytes.  The resulting k order inside the group (position pos holds k = 4 (pos & 3) + ORDER[pos >> 2])
//   is what the decode produces cheapest; the activations are written to shared memory in the same order, which
//   leaves every product, and the sum, unchanged.
//
// Roles (512 threads, one CTA per SM, persistent over 128-row tiles): warp 0 streams [128 rows x 256 k] code tiles
// and their scale tiles (TMA, started before the grid-dependency wait: weights do not depend on the previous
// kernel); warp 1 owns the tensor memory and one of its lanes issues the MMAs; warps 1..7 write the activations
// (16 B columns, tokens beyond M zero) into shared memory after the dependency wait; warps 4..7 are the epilogue
// (one tensor-memory subpartition each); warps 8..15 decode, in two sets taking alternate 256-k chunks, each
// thread one row of the tile.  A chunk's decoded weights fill one of the 128-column A buffers; the MMA lane
// consumes them with 16 MMAs of K = 16, spread over several 16-column accumulators.  Every wait is bounded; a failed
// wait records an error and the kernel still drains its copies and releases its tensor memory.
#pragma once
#include <cuda.h>

#include "fp4x_common.cuh"
#include "fp4x_tc.cuh"

namespace fp4x {
namespace tc {

constexpr int kI2Sets = 2;                          // decoder sets (4 warps each)
constexpr int kI2Threads = 256 + 128 * kI2Sets;     // 8 role warps + the decoders
constexpr int kI2KC = 256;                          // k per chunk
constexpr int kI2MaxStages = 12;
#ifndef FP4X_I2_ACC
#define FP4X_I2_ACC 4
#endif
#ifndef FP4X_I2_DBUFS
#define FP4X_I2_DBUFS 2
#endif
#ifndef FP4X_I2_ABUFS
#define FP4X_I2_ABUFS 3
#endif
// Consecutive MMAs of a chunk go to kI2Acc different accumulators: MMAs into one accumulator run one after the
// other, and at N = 16 their latency, not their arithmetic, would set the pace.  The accumulator sets are
// double-buffered across tiles (kI2DBufs), so the epilogue of a tile overlaps the MMAs of the next.
constexpr int kI2Acc = FP4X_I2_ACC;
constexpr int kI2DBufs = FP4X_I2_DBUFS;
constexpr int kI2Bufs = FP4X_I2_ABUFS;              // A buffers in tensor memory: 128 columns each (256 k of bf16)
constexpr int kI2ColD = 0;                          // kI2DBufs x kI2Acc accumulators of 16 columns
constexpr int kI2ColA = 512 - 128 * kI2Bufs;
static_assert(kI2DBufs * kI2Acc * 16 <= kI2ColA, "tensor-memory columns");
constexpr int kI2CodeBytes = kRows * kI2KC / 4;     // 8 KB of codes per chunk: [128 rows][64 bytes], 64-byte swizzle
constexpr int kI2StageBytes = 12 * 1024;            // codes + up to [128 rows][32 bytes] of fp16 scales
constexpr int kI2N = 16;                            // MMA N: tokens, zero-padded
constexpr int kI2MaxM = 16;

struct I2Args {
  CUtensorMap tm;    // codes [N rows][K/4 bytes] u8, box {64 bytes, 128 rows}, 64-byte swizzle
  CUtensorMap tms;   // scales [N rows][2K/g bytes] u8, box {512/g bytes, 128 rows}, no swizzle
  const __nv_bfloat16* x;
  int64_t x_stride;
  void* out;
  void* out_bf16;    // optional bf16 copy of the output
  int64_t out_stride;
  int out_dtype;
  int M, N, K, group;
  int tiles;         // ceil(N / 128)
  int NS;
  int smem_b, smem_misc;
  int* err;
  unsigned long long* tl;  // launch timeline record (diagnostic) or null
};

FP4X_DEV uint32_t idesc_bf16_n16() {
  // kind::f16: D f32 (bits 4-5 = 1), A bf16 (bits 7-9 = 1), B bf16 (bits 10-12 = 1), both K-major, N = 16, M = 128
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kI2N >> 3) << 17) | (8u << 24);
}
// D (tensor memory) += A (tensor memory) x B (shared memory descriptor)
FP4X_DEV void mma_bf16_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Eight bf16 pairs of one 16-k group: register 2p + h holds the weights of bytes 2h, 2h + 1 at bit pair p.
FP4X_DEV void int2_group_bf16(uint32_t w, uint32_t tlo, uint32_t thi, uint32_t* o) {
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t z = (w >> (2 * p)) & 0x03030303u;
    const uint32_t sl = z * 0x11u + 0x4040u;                 // nibbles z0, z0 + 4, z1, z1 + 4
    const uint32_t sh = __umulhi(z, 0x110000u) + 0x4040u;    // nibbles z2, z2 + 4, z3, z3 + 4
    o[2 * p] = prmt(tlo, thi, sl);
    o[2 * p + 1] = prmt(tlo, thi, sh);
  }
}

// byte offset of (B row n, k position kp) in the 128-byte-swizzled K-major B operand: 64-k slabs of 16 rows
FP4X_DEV uint32_t i2_b_offset(int n, int kp) {
  const int slab = kp >> 6, byte = (kp & 63) * 2;
  const int r = n & 7, chunk = byte >> 4;
  return (uint32_t)(slab * 2048 + (n >> 3) * 1024 + r * 128 + ((chunk ^ r) << 4) + (byte & 15));
}

__global__ void __launch_bounds__(kI2Threads, 1) int2_tc_kernel(const __grid_constant__ I2Args A) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cpt = A.K / kI2KC;  // chunks per tile
  const int my_tiles = A.tiles > (int)blockIdx.x ? (A.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 0;
  const int nq = my_tiles * cpt;  // chunks of this CTA
  const int sc_bytes = 512 / A.group;  // scale bytes per row per chunk (32 for g16, 16 for g32)

  uint64_t* bars = reinterpret_cast<uint64_t*>(base + A.smem_misc);
  const uint32_t full0 = smem_u32(bars), empty0 = full0 + 8 * kI2MaxStages;
  const uint32_t afull0 = empty0 + 8 * kI2MaxStages, aempty0 = afull0 + 8 * kI2Bufs;
  const uint32_t dfull0 = aempty0 + 8 * kI2Bufs, dempty0 = dfull0 + 8 * kI2DBufs;
  uint32_t* tmem_slot =
      reinterpret_cast<uint32_t*>(base + A.smem_misc + 8 * (2 * kI2MaxStages + 2 * kI2Bufs + 2 * kI2DBufs));

  if (threadIdx.x == 0) {
    for (int s = 0; s < A.NS; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 4);  // the four warps of the decoder set that read the stage
    }
    for (int b = 0; b < kI2Bufs; ++b) {
      mbar_init(afull0 + 8 * b, 4);  // the four decoder warps wrote their 32 rows each
      mbar_init(aempty0 + 8 * b, 1);  // tcgen05.commit: the MMAs reading the buffer are done
    }
    for (int b = 0; b < kI2DBufs; ++b) {
      mbar_init(dfull0 + 8 * b, 1);
      mbar_init(dempty0 + 8 * b, 4);  // the four epilogue warps read the accumulator
    }
    mbar_init_fence();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- producer: code tiles and scale tiles ----------------
    pdl_launch_dependents();
    int issued = 0;
    for (int q = 0; q < nq && ok; ++q) {
      const int s = q % A.NS, round = q / A.NS;
      if (round > 0 && !mbar_wait_bounded(empty0 + 8 * s, (uint32_t)((round - 1) & 1), A.err)) { ok = false; break; }
      const int tile = (int)blockIdx.x + (q / cpt) * (int)gridDim.x, c = q % cpt;
      if (lane == 0) {
        const uint32_t stage = smem_u32(base) + (uint32_t)s * kI2StageBytes;
        mbar_arrive_expect_tx(full0 + 8 * s, (uint32_t)(kI2CodeBytes + kRows * sc_bytes));
        tma_load_2d(stage, &A.tm, c * (kI2KC / 4), tile * kRows, full0 + 8 * s);
        tma_load_2d(stage + kI2CodeBytes, &A.tms, c * sc_bytes, tile * kRows, full0 + 8 * s);
      }
      issued = q + 1;
    }
    // no copy may still be landing when the CTA exits: wait for the last use of every stage (bounded)
    for (int q = max(0, issued - A.NS); q < issued; ++q)
      mbar_wait_bounded(full0 + 8 * (q % A.NS), (uint32_t)((q / A.NS) & 1), A.err);
  } else if (warp >= 8) {
    // ---------------- decoders: set `set` takes chunks q = set, set + kI2Sets, ... ----------------
    const int set = (warp - 8) >> 2, sub = warp & 3;
    const int r = 32 * sub + lane;  // row of the tile
    const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16);
    for (int q = set; q < nq && ok; q += kI2Sets) {
      const int s = q % A.NS, b = q % kI2Bufs;
      if (!mbar_wait_bounded(full0 + 8 * s, (uint32_t)((q / A.NS) & 1), A.err)) { ok = false; break; }
      if (q >= kI2Bufs && !mbar_wait_bounded(aempty0 + 8 * b, (uint32_t)(((q / kI2Bufs) - 1) & 1), A.err)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t stage = smem_u32(base) + (uint32_t)s * kI2StageBytes;
      const uint32_t crow = stage + (uint32_t)r * 64u;
      const uint32_t srow = stage + kI2CodeBytes + (uint32_t)(r * sc_bytes);
      const uint32_t abuf = trow + kI2ColA + 128u * (uint32_t)b;
      uint32_t sw[8];  // this chunk's scales of the row: 16 (g16) or 8 (g32) fp16
      {
        const uint4 s0 = lds128(srow);
        sw[0] = s0.x; sw[1] = s0.y; sw[2] = s0.z; sw[3] = s0.w;
        if (A.group == 16) {
          const uint4 s1 = lds128(srow + 16);
          sw[4] = s1.x; sw[5] = s1.y; sw[6] = s1.z; sw[7] = s1.w;
        } else {
          sw[4] = sw[5] = sw[6] = sw[7] = 0u;
        }
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) {  // 64 k: 16 code bytes = 4 groups of 16
        const uint4 cw = lds128(crow + (uint32_t)(((h ^ ((r >> 1) & 3)) << 4)));
        const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
        uint32_t v[16];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int gq = 4 * h + i;  // 16-group of the chunk
          uint32_t s16;
          if (A.group == 16) s16 = (sw[gq >> 1] >> (16 * (gq & 1))) & 0xffffu;
          else s16 = (sw[gq >> 2] >> (16 * ((gq >> 1) & 1))) & 0xffffu;
          uint32_t tlo, thi;
          int2_table(s16, tlo, thi);
          int2_group_bf16(words[i], tlo, thi, v + 8 * (i & 1));
          if (i & 1) tc_st16(abuf + 32u * h + 16u * (i >> 1), v);
        }
      }
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(empty0 + 8 * s);
        mbar_arrive(afull0 + 8 * b);
      }
    }
  } else {
    // ---------------- warps 1..7: activations into the B operand (after the grid-dependency wait) -------------
    const int tid = threadIdx.x - 32, nthr = 224;
    pdl_wait();
    uint8_t* bsm = base + A.smem_b;
    const int groups = A.K / 16;
    for (int idx = tid; idx < kI2N * groups; idx += nthr) {
      const int n = idx / groups, g = idx - n * groups;
      uint32_t in[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (n < A.M) {
        const uint4* src = reinterpret_cast<const uint4*>(A.x + (int64_t)n * A.x_stride + 16 * g);
        const uint4 a0 = src[0], a1 = src[1];
        in[0] = a0.x; in[1] = a0.y; in[2] = a0.z; in[3] = a0.w;
        in[4] = a1.x; in[5] = a1.y; in[6] = a1.z; in[7] = a1.w;
      }
      // position pos of the group holds k = 4 (pos & 3) + ORDER[pos >> 2]
      uint4 o0, o1;
      o0.x = prmt(in[0], in[2], 0x5410u); o0.y = prmt(in[4], in[6], 0x5410u);
      o0.z = prmt(in[1], in[3], 0x5410u); o0.w = prmt(in[5], in[7], 0x5410u);
      o1.x = prmt(in[0], in[2], 0x7632u); o1.y = prmt(in[4], in[6], 0x7632u);
      o1.z = prmt(in[1], in[3], 0x7632u); o1.w = prmt(in[5], in[7], 0x7632u);
      *reinterpret_cast<uint4*>(bsm + i2_b_offset(n, 16 * g)) = o0;
      *reinterpret_cast<uint4*>(bsm + i2_b_offset(n, 16 * g + 8)) = o1;
    }
    fence_proxy_async_smem();  // the tensor core reads B through the async proxy
    named_bar(1, nthr);
    if (warp == 1) {
      // ---------------- MMA issue (lane 0) ----------------
      if (lane == 0) {
        const uint32_t idesc = idesc_bf16_n16();
        const uint32_t bbase = smem_u32(bsm);
        for (int q = 0; q < nq && ok; ++q) {
          const int lt = q / cpt, c = q % cpt, b = q % kI2Bufs, db = lt % kI2DBufs, u = lt / kI2DBufs;
          if (c == 0 && lt >= kI2DBufs && !mbar_wait_bounded(dempty0 + 8 * db, (uint32_t)((u - 1) & 1), A.err)) {
            ok = false;
            break;
          }
          if (!mbar_wait_bounded(afull0 + 8 * b, (uint32_t)((q / kI2Bufs) & 1), A.err)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < kI2KC / 16; ++j) {
            const int kp = c * kI2KC + 16 * j;  // k position of the MMA's first column
            const uint64_t bdesc = smem_desc_sw128(bbase + (uint32_t)((kp >> 6) * 2048 + ((kp & 63) >> 4) * 32));
            mma_bf16_ts(tmem + kI2ColD + 16u * (uint32_t)(db * kI2Acc + j % kI2Acc),
                        tmem + kI2ColA + 128u * (uint32_t)b + 8u * (uint32_t)j, bdesc, idesc,
                        (c > 0 || j >= kI2Acc) ? 1u : 0u);
          }
          tc_commit(aempty0 + 8 * b);
          if (c == cpt - 1) tc_commit(dfull0 + 8 * db);
        }
      }
      __syncwarp();
    } else if (warp >= 4) {
      // ---------------- epilogue: row 32 sub + lane of each tile, tokens 0..M-1 ----------------
      const int sub = warp & 3;
      const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16);
      for (int lt = 0; lt < my_tiles && ok; ++lt) {
        const int db = lt % kI2DBufs;
        if (!mbar_wait_bounded(dfull0 + 8 * db, (uint32_t)((lt / kI2DBufs) & 1), A.err)) { ok = false; break; }
        tc_fence_after();
        float d[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) d[i] = 0.f;
#pragma unroll
        for (int a = 0; a < kI2Acc; ++a) {  // accumulators summed in a fixed order
          uint32_t q16[16];
          tc_ld16(trow + kI2ColD + 16u * (uint32_t)(db * kI2Acc + a), q16);
          tc_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) d[i] += __uint_as_float(q16[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(dempty0 + 8 * db);
        const int row = ((int)blockIdx.x + lt * (int)gridDim.x) * kRows + 32 * sub + lane;
        if (row < A.N) {
#pragma unroll
          for (int m = 0; m < kI2MaxM; ++m) {
            if (m < A.M) {
              const float val = d[m];
              store_out(A.out, A.out_dtype, (int64_t)m * A.out_stride + row, val);
              if (A.out_bf16)
                reinterpret_cast<__nv_bfloat16*>(A.out_bf16)[(int64_t)m * A.out_stride + row] = __float2bfloat16_rn(val);
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

}  // namespace tc
}  // namespace fp4x
