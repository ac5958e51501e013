// Decode-shaped (M <= 16) quantized GEMV core for sm_100a.
//
//   out[m, n] = sum_k x[m, k] * W[n, k]      x: bf16 [M, K];  W: packed rows in one of six formats
//
// Structure (up to two CTAs per SM; each CTA = 4 consumer warps + 1 producer warp):
//   * Work unit = (block of 64 weight rows) x (k chunk of KC elements).  K is cut into KP panels (grid.y); inside a
//     panel the RT*NCH units are split evenly over the CPP CTAs of the panel (stream-K), so every CTA streams the
//     same number of bytes.  A row block shared by several CTAs or panels is combined by the last arriving warp,
//     which sums the partial slots in a fixed order (deterministic) and resets its arrival counter to zero.
//   * The producer warp streams each unit into a ring of shared-memory stages with 2D TMA loads
//     (cp.async.bulk.tensor, box = {64 or 128 bytes, 64 rows}, 64B/128B swizzle: one 4-8 KB request per box),
//     plus 16/8/4-byte cp.async copies of the scale rows.  It starts before griddepcontrol.wait: weights never
//     depend on the previous kernel, so under programmatic dependent launch the first stages are already in
//     flight while the previous kernel drains.
//   * The panel's activations are staged once per CTA in shared memory, permuted into the mma B-fragment order of
//     the format and converted to f16 with a per-(token, panel) power-of-two scale (exact for every element within
//     2^31 of the token's panel maximum) or kept as bf16.
//   * Each consumer warp owns 16 rows of the stage.  A fragments come straight from the swizzled tiles with
//     ldmatrix (bank-conflict free), are decoded in registers with exact conversions (fp8/fp4 -> f16 cvt, int8/
//     int6 -> f16 magic-number adds, INT2 -> bf16 via a per-group byte-permute table) and multiplied on the tensor
//     cores (mma.sync m16n8k16, fp32 accumulate).  Per-group scales are applied to the fp32 group partials
//     (deferred) for the fp8/int formats, so products stay exact.
#pragma once
#include <cuda.h>

#include "fp4x_common.cuh"

namespace fp4x {

constexpr int kRW = 4;                           // row warps: 16 rows each, one 64-row block
constexpr int kKG = 2;                           // k-groups: each stage's chunks are split between two warp sets
constexpr int kCWarps = kRW * kKG;               // consumer warps
constexpr int kThreads = (kCWarps + 1) * 32;     // + one producer warp
constexpr int kRB = 16 * kRW;                    // rows per stage
constexpr int kMaxStages = 8;

enum Fmt : int { FMT_MX8 = 0, FMT_W8 = 1, FMT_W6 = 2, FMT_NV4 = 3, FMT_BF16 = 4, FMT_INT2 = 5 };
enum Epi : int { EPI_STORE = 0, EPI_HC_DOWN = 1, EPI_HC_UP = 2, EPI_HEAD = 3 };

// per-format geometry; bytes-per-k values are num/den
struct FmtGeom {
  int kq;         // k per 16-byte chunk of plane 0
  int n0, d0;     // plane-0 bytes per k
  int n1, d1;     // plane-1 bytes per k (0 if absent)
  int sn, sd;     // scale bytes per k (INT2: sd = group / 2)
  int qb;         // activation staging block (consecutive k)
  int xf16;       // activations converted to scaled f16 (else kept bf16)
  int kmin;       // k granularity of a stage (one decode block of 64 or 128 plane-0 bytes)
};

__host__ __device__ constexpr FmtGeom fmt_geom(int fmt) {
  return fmt == FMT_MX8    ? FmtGeom{16, 1, 1, 0, 1, 1, 32, 4, 1, 64}
         : fmt == FMT_W8   ? FmtGeom{16, 1, 1, 0, 1, 1, 16, 4, 0, 64}
         : fmt == FMT_W6   ? FmtGeom{32, 1, 2, 1, 4, 1, 16, 8, 0, 256}
         : fmt == FMT_NV4  ? FmtGeom{32, 1, 2, 0, 1, 1, 16, 4, 1, 128}
         : fmt == FMT_BF16 ? FmtGeom{8, 2, 1, 0, 1, 0, 1, 16, 0, 32}
                           : FmtGeom{64, 1, 4, 0, 1, 1, 8, 16, 0, 256};  // INT2 (scale sd set at runtime)
}

struct GemvItem {
  const void* x;        // bf16 [M, K] (row stride x_stride elements)
  const uint8_t* sc;    // scales
  void* out;            // primary output
  void* out2;           // HC down: bottleneck output; head: bf16 copy of the logits
};

// one entry of a batched launch: the TMA descriptor of the codes plus the pointers of the item
struct alignas(64) BatchEntry {
  CUtensorMap tm0;
  const void* x;
  const uint8_t* sc;
  void* out;
  void* pad;
};

struct alignas(64) GemvArgs {
  CUtensorMap tm0;        // plane-0 codes [N, ld0] uint8, box {BI0, 64}
  CUtensorMap tm1;        // plane-1 codes (W6 high bit pairs), box {BI1, 64}
  GemvItem item;          // the matrix of a single call
  const BatchEntry* batch;  // batched W8: one entry per grid.z (device memory), or null
  int M, N, K;
  int64_t x_stride;
  int64_t lds;            // scale row stride (bytes)
  int64_t out_stride;     // elements between tokens of out (and out2 for the head)
  int out_dtype;
  float post;             // multiplier on the final sum (NVFP4 global scale)
  int KPW, KP;            // panel width and count
  int KC, NCH;            // chunk width (k) and chunks per (row block, panel)
  int CPP;                // CTAs per (panel, batch item)
  int RT;                 // row blocks
  int NS;                 // stages
  int SMAX;               // partial slots per (batch, panel, row block) when KP > 1
  int whole;              // 1: CTAs own whole row blocks (all NCH chunks)
  int group;              // INT2 scale group (16 or 32)
  int BI0, BI1;           // TMA box inner bytes of the planes (64 or 128)
  int NB0;                // plane-0 boxes per stage
  int SB;                 // scale bytes per row per stage
  int scw;                // scale copy width (4, 8 or 16 bytes)
  int STG;                // stage bytes (multiple of 1024)
  int off_p1, off_sc;     // offsets of plane 1 and of the scales inside a stage
  int XP;                 // activation token pitch (bytes)
  int smem_x, smem_misc, smem_scr;  // offsets of the regions after the 1024-aligned base (stages start at 0)
  int smem_xraw;          // raw bf16 activation panel [M][KPW] (bulk-copied after griddepcontrol.wait)
  int smem_comb;          // k-group hand-over of partial sums: [kRW][32 lanes][NT * 4] fp32
  int cluster;            // > 1: the KP panel CTAs of a row block form a cluster and reduce through its leader
  int smem_red;           // cluster leader: partial sums of the other panels [cluster - 1][kRW][32][NT * 4] fp32
  int lr, hc, bj;         // hyper-connection epilogues
  const void* nrm;        // HC up: normalized input [M, hc*H]
  int64_t nrm_stride;
  float* ws;              // partial slots
  int* sem;               // arrival counters [batch * RT * 4], zero on entry and on exit
  int* err;               // device error word
  int xdirect;            // 1: no raw panel in shared memory; staging reads the activations from global memory
  unsigned long long* tl;  // launch timeline record (diagnostic) or null
};

// ------------------------------------------------------------------------------------------------------
// work partition helpers (identical on host and device)
// ------------------------------------------------------------------------------------------------------
__host__ __device__ inline int64_t range_begin(int64_t U, int W, int w) { return U * w / W; }
// the part that owns unit u when U units are split over W parts by range_begin
__host__ __device__ inline int owner_of(int64_t u, int64_t U, int W) { return (int)(((u + 1) * W + U - 1) / U) - 1; }

// fetch-and-add with acquire-release semantics at GPU scope
FP4X_DEV int atomic_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// ------------------------------------------------------------------------------------------------------
// TMA, async copies, ldmatrix
// ------------------------------------------------------------------------------------------------------
FP4X_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(tm), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
FP4X_DEV void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
FP4X_DEV void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
FP4X_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
FP4X_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
FP4X_DEV void named_bar(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

// physical offset of logical byte `off` inside a tile written by TMA with the 64B/128B swizzle of box inner BI
FP4X_DEV uint32_t swz(uint32_t off, int BI) {
  const uint32_t mask = BI == 128 ? 7u : 3u;
  return off ^ (((off >> 7) & mask) << 4);
}

// ------------------------------------------------------------------------------------------------------
// activation staging: permuted B-fragment order, one quad (4 k values) per (token, step, tq)
// ------------------------------------------------------------------------------------------------------
// For a staging block kb (qb consecutive k of the panel) of format FMT: the steps of its quads and the tq.
template <int FMT>
FP4X_DEV void stage_block_positions(int kb, int (&s)[4], int& tq) {
  if (FMT == FMT_MX8) {  // k0 = 32G + 16h + 4tq
    s[0] = 2 * (kb >> 3) + ((kb >> 2) & 1);
    tq = kb & 3;
  } else if (FMT == FMT_W8) {  // k0 = 64G + 16h + 4tq
    s[0] = 4 * (kb >> 4) + ((kb >> 2) & 3);
    tq = kb & 3;
  } else if (FMT == FMT_NV4) {  // k0 = 32C + 8tq + 4h
    s[0] = 2 * (kb >> 3) + (kb & 1);
    tq = (kb >> 1) & 3;
  } else if (FMT == FMT_W6) {  // k0 = 32G + 8tq: two quads
    s[0] = 2 * (kb >> 2);
    s[1] = s[0] + 1;
    tq = kb & 3;
  } else if (FMT == FMT_BF16) {  // one 16-k step: four quads, one per tq
    s[0] = kb;
    tq = 0;
  } else {  // INT2: one 16-k group kb = 4C + tq: four quads (steps 4C + p)
    const int base = 4 * (kb >> 2);
    s[0] = base;
    s[1] = base + 1;
    s[2] = base + 2;
    s[3] = base + 3;
    tq = kb & 3;
  }
}

FP4X_DEV uint32_t cvt_pair(uint32_t bf2, float scl, bool xf16) {
  if (!xf16) return bf2;
  const float lo = bf16_bits_to_f32(bf2 & 0xffffu) * scl;
  const float hi = bf16_bits_to_f32(bf2 >> 16) * scl;
  return pack_f16x2(lo, hi);
}
// two 16-bit values (halves lo_idx of lo_src and hi_idx of hi_src) in one word
FP4X_DEV uint32_t pick2(uint32_t lo_src, int lo_idx, uint32_t hi_src, int hi_idx) {
  const uint32_t a = (lo_src >> (16 * lo_idx)) & 0xffffu;
  const uint32_t b = (hi_src >> (16 * hi_idx)) & 0xffffu;
  return a | (b << 16);
}

// The conversion passes of the activation staging over a raw bf16 panel in global memory (rows xrs elements apart):
// 16-token plans whose raw panel would not fit in shared memory beside the converted panel and the weight stages.
// The shared-memory path in stage_activations keeps its own copy of the same passes: routing it through this
// function changed the code of the M <= 8 kernels and cost 0.5-1% of the decode step (measured).
template <int FMT>
FP4X_DEV void stage_convert(const GemvArgs& A, uint8_t* base, int MP, const __nv_bfloat16* xr, int64_t xrs) {
  constexpr FmtGeom G = fmt_geom(FMT);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int nthr = kCWarps * 32;
  float* xsc = reinterpret_cast<float*>(base + A.smem_misc);  // [MP] scale, [MP] inverse
  const int KPW = A.KPW;
  if (G.xf16) {
    for (int tok = warp; tok < MP; tok += kCWarps) {
      float mx = 0.f;
      if (tok < A.M) {
        const uint4* row = reinterpret_cast<const uint4*>(xr + (int64_t)tok * xrs);
        for (int i = lane; i < KPW / 8; i += 32) {
          const uint4 v = row[i];
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            mx = fmaxf(mx, fabsf(bf16_bits_to_f32(w[e] & 0xffffu)));
            mx = fmaxf(mx, fabsf(bf16_bits_to_f32(w[e] >> 16)));
          }
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) {
        int t = 0;
        const uint32_t bits = __float_as_uint(mx);
        if (mx > 0.f && (bits >> 23) < 255u) {
          const int e = (int)(bits >> 23) - 127;  // exponent of the maximum (subnormals count as -127)
          t = 14 - e;
          t = t < -113 ? -113 : (t > 126 ? 126 : t);
        }
        xsc[tok] = __uint_as_float((uint32_t)(127 + t) << 23);
        xsc[MP + tok] = __uint_as_float((uint32_t)(127 - t) << 23);
      }
    }
    named_bar(1, nthr);
  }
  // Only the M real token rows are converted: B columns >= M are never written, and since each column of an MMA
  // result depends on its own B column alone, whatever they hold reaches only output columns that are not stored.
  const uint32_t xbase = smem_u32(base + A.smem_x);
  const int nblk = KPW / G.qb;
  for (int tok = 0; tok < A.M; ++tok)
  for (int kb = tid; kb < nblk; kb += nthr) {
    const float scl = G.xf16 ? xsc[tok] : 1.f;
    uint32_t v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    {
      const __nv_bfloat16* src = xr + (int64_t)tok * xrs + kb * G.qb;
      if (G.qb == 4) {
        const uint2 t = *reinterpret_cast<const uint2*>(src);
        v[0] = t.x; v[1] = t.y;
      } else if (G.qb == 8) {
        const uint4 t = *reinterpret_cast<const uint4*>(src);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
        const uint4 t0 = *reinterpret_cast<const uint4*>(src);
        const uint4 t1 = *reinterpret_cast<const uint4*>(src + 8);
        v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
        v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
      }
    }
    int s[4];
    int tq;
    stage_block_positions<FMT>(kb, s, tq);
    const uint32_t trow = xbase + tok * A.XP;
    if (G.qb == 4) {
      sts64(trow + s[0] * 32 + tq * 8, cvt_pair(v[0], scl, G.xf16), cvt_pair(v[1], scl, G.xf16));
    } else if (G.qb == 8) {
      // W6: elements r0..r7 (two per word); quads (r0,r4,r1,r5) and (r2,r6,r3,r7)
      sts64(trow + s[0] * 32 + tq * 8, cvt_pair(pick2(v[0], 0, v[2], 0), scl, G.xf16),
            cvt_pair(pick2(v[0], 1, v[2], 1), scl, G.xf16));
      sts64(trow + s[1] * 32 + tq * 8, cvt_pair(pick2(v[1], 0, v[3], 0), scl, G.xf16),
            cvt_pair(pick2(v[1], 1, v[3], 1), scl, G.xf16));
    } else if (FMT == FMT_BF16) {
      // one step of 16 k: quad q = (e[2q], e[2q+1], e[8+2q], e[9+2q]) = words v[q], v[4+q]
#pragma unroll
      for (int q = 0; q < 4; ++q) sts64(trow + s[0] * 32 + q * 8, v[q], v[4 + q]);
    } else {
      // INT2: elements e0..e15 of one group; quad p = (ORDER[p] + 4j), ORDER = (0,2,1,3)
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int o = (p == 1) ? 2 : (p == 2 ? 1 : p);
        const int e0 = o, e1 = 4 + o, e2 = 8 + o, e3 = 12 + o;
        const uint32_t lo = pick2(v[e0 >> 1], e0 & 1, v[e1 >> 1], e1 & 1);
        const uint32_t hi = pick2(v[e2 >> 1], e2 & 1, v[e3 >> 1], e3 & 1);
        sts64(trow + s[p] * 32 + tq * 8, cvt_pair(lo, scl, G.xf16), cvt_pair(hi, scl, G.xf16));
      }
    }
  }
}

template <int FMT, int NT>
FP4X_DEV void stage_activations(const GemvArgs& A, const GemvItem& it, uint8_t* base, int MP, int k_panel0,
                                uint32_t xbar) {
  if constexpr (FMT == FMT_W8) {
    // W8 reads bf16 activations in their own order (stage_block_positions is the identity: block kb at byte 8 kb),
    // so the operand panel is the raw token rows at the padded pitch XP: the bulk copies land there directly and
    // nothing is converted
    if (threadIdx.x == 0) {
      const uint32_t bytes = (uint32_t)A.KPW * 2u;
      mbar_arrive_expect_tx(xbar, bytes * (uint32_t)A.M);
      const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(it.x);
      for (int m = 0; m < A.M; ++m)
        bulk_g2s(smem_u32(base + A.smem_x) + m * A.XP, x + (int64_t)m * A.x_stride + k_panel0, bytes, xbar);
    }
    const bool landed = mbar_wait_bounded(xbar, 0, A.err);
    FP4X_TL(if (landed && threadIdx.x == 0) tl_last(A.tl, kTlXLanded));
    (void)landed;
    return;
  }
  // 16-token plans may leave the raw panel in global memory (the flag is compiled into those kernels only)
  if constexpr (NT == 2) {
    if (A.xdirect) {
      stage_convert<FMT>(A, base, MP, reinterpret_cast<const __nv_bfloat16*>(it.x) + k_panel0, A.x_stride);
      return;
    }
  }
  constexpr FmtGeom G = fmt_geom(FMT);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int nthr = kCWarps * 32;
  float* xsc = reinterpret_cast<float*>(base + A.smem_misc);  // [MP] scale, [MP] inverse
  const int KPW = A.KPW;
  // one bulk copy per token row brings the raw panel into shared memory in a single round trip
  const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(base + A.smem_xraw);
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)KPW * 2u;
    mbar_arrive_expect_tx(xbar, bytes * (uint32_t)A.M);
    const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(it.x);
    for (int m = 0; m < A.M; ++m)
      bulk_g2s(smem_u32(base + A.smem_xraw) + m * bytes, x + (int64_t)m * A.x_stride + k_panel0, bytes, xbar);
  }
  if (!mbar_wait_bounded(xbar, 0, A.err)) return;
  FP4X_TL(if (tid == 0) tl_last(A.tl, kTlXLanded));
  if (G.xf16) {
    for (int tok = warp; tok < MP; tok += kCWarps) {
      float mx = 0.f;
      if (tok < A.M) {
        const uint4* row = reinterpret_cast<const uint4*>(xr + (int64_t)tok * KPW);
        for (int i = lane; i < KPW / 8; i += 32) {
          const uint4 v = row[i];
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            mx = fmaxf(mx, fabsf(bf16_bits_to_f32(w[e] & 0xffffu)));
            mx = fmaxf(mx, fabsf(bf16_bits_to_f32(w[e] >> 16)));
          }
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) {
        int t = 0;
        const uint32_t bits = __float_as_uint(mx);
        if (mx > 0.f && (bits >> 23) < 255u) {
          const int e = (int)(bits >> 23) - 127;  // exponent of the maximum (subnormals count as -127)
          t = 14 - e;
          t = t < -113 ? -113 : (t > 126 ? 126 : t);
        }
        xsc[tok] = __uint_as_float((uint32_t)(127 + t) << 23);
        xsc[MP + tok] = __uint_as_float((uint32_t)(127 - t) << 23);
      }
    }
    named_bar(1, nthr);
  }
  // Only the M real token rows are converted: B columns >= M are never written, and since each column of an MMA
  // result depends on its own B column alone, whatever they hold reaches only output columns that are not stored.
  const uint32_t xbase = smem_u32(base + A.smem_x);
  const int nblk = KPW / G.qb;
  for (int tok = 0; tok < A.M; ++tok)
  for (int kb = tid; kb < nblk; kb += nthr) {
    const float scl = G.xf16 ? xsc[tok] : 1.f;
    uint32_t v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    {
      const __nv_bfloat16* src = xr + (int64_t)tok * KPW + kb * G.qb;
      if (G.qb == 4) {
        const uint2 t = *reinterpret_cast<const uint2*>(src);
        v[0] = t.x; v[1] = t.y;
      } else if (G.qb == 8) {
        const uint4 t = *reinterpret_cast<const uint4*>(src);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
        const uint4 t0 = *reinterpret_cast<const uint4*>(src);
        const uint4 t1 = *reinterpret_cast<const uint4*>(src + 8);
        v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
        v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
      }
    }
    int s[4];
    int tq;
    stage_block_positions<FMT>(kb, s, tq);
    const uint32_t trow = xbase + tok * A.XP;
    if (G.qb == 4) {
      sts64(trow + s[0] * 32 + tq * 8, cvt_pair(v[0], scl, G.xf16), cvt_pair(v[1], scl, G.xf16));
    } else if (G.qb == 8) {
      // W6: elements r0..r7 (two per word); quads (r0,r4,r1,r5) and (r2,r6,r3,r7)
      sts64(trow + s[0] * 32 + tq * 8, cvt_pair(pick2(v[0], 0, v[2], 0), scl, G.xf16),
            cvt_pair(pick2(v[0], 1, v[2], 1), scl, G.xf16));
      sts64(trow + s[1] * 32 + tq * 8, cvt_pair(pick2(v[1], 0, v[3], 0), scl, G.xf16),
            cvt_pair(pick2(v[1], 1, v[3], 1), scl, G.xf16));
    } else if (FMT == FMT_BF16) {
      // one step of 16 k: quad q = (e[2q], e[2q+1], e[8+2q], e[9+2q]) = words v[q], v[4+q]
#pragma unroll
      for (int q = 0; q < 4; ++q) sts64(trow + s[0] * 32 + q * 8, v[q], v[4 + q]);
    } else {
      // INT2: elements e0..e15 of one group; quad p = (ORDER[p] + 4j), ORDER = (0,2,1,3)
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int o = (p == 1) ? 2 : (p == 2 ? 1 : p);
        const int e0 = o, e1 = 4 + o, e2 = 8 + o, e3 = 12 + o;
        const uint32_t lo = pick2(v[e0 >> 1], e0 & 1, v[e1 >> 1], e1 & 1);
        const uint32_t hi = pick2(v[e2 >> 1], e2 & 1, v[e3 >> 1], e3 & 1);
        sts64(trow + s[p] * 32 + tq * 8, cvt_pair(lo, scl, G.xf16), cvt_pair(hi, scl, G.xf16));
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------------
// per-format stage compute: one warp, 16 rows, one stage
// ------------------------------------------------------------------------------------------------------
struct WarpCtx {
  uint32_t p0, p1, sc;  // shared addresses of the stage planes and scales
  int BI0, BI1, NB0, SB, CPB;
  uint32_t lrow0;       // ldmatrix: this lane's row offset inside a box (row * BI0)
  int lswz, lsel;       // ldmatrix: this lane's swizzle key and chunk select (0/1)
  uint32_t xb;          // activation address of step 0 of this stage for token row g and tq
  int XP;
  int g, tq, rbase;     // rbase = 16 * warp (first row of the warp inside the stage)
  int gshift;           // INT2: 1 when scale groups are 32
};

template <int NT>
FP4X_DEV void load_b(const WarpCtx& c, int s, uint32_t (&b0)[NT], uint32_t (&b1)[NT]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const uint2 v = lds64(c.xb + t * 8 * c.XP + s * 32);
    b0[t] = v.x;
    b1[t] = v.y;
  }
}

// chunks (chunk, chunk+1) x (rows g, g+8) of plane 0, box b: r0 = (g, chunk), r1 = (g+8, chunk),
// r2 = (g, chunk+1), r3 = (g+8, chunk+1); each register = bytes 4tq..4tq+3 of that 16-byte row chunk
FP4X_DEV void ld_pair(const WarpCtx& c, int b, int chunk, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  const uint32_t addr =
      c.p0 + (uint32_t)b * (uint32_t)(kRB * c.BI0) + c.lrow0 + 16u * (uint32_t)((chunk + c.lsel) ^ c.lswz);
  ldsm_x4(addr, r0, r1, r2, r3);
}

template <int NT>
FP4X_DEV void zero4(float (&a)[NT][4]) {
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) a[t][e] = 0.f;
}

template <int NT>
FP4X_DEV void fma_scaled(float (&acc)[NT][4], const float (&tmp)[NT][4], float s_lo, float s_hi) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    acc[t][0] = fmaf(tmp[t][0], s_lo, acc[t][0]);
    acc[t][1] = fmaf(tmp[t][1], s_lo, acc[t][1]);
    acc[t][2] = fmaf(tmp[t][2], s_hi, acc[t][2]);
    acc[t][3] = fmaf(tmp[t][3], s_hi, acc[t][3]);
  }
}

template <int NT>
FP4X_DEV void mma_f16_acc(float (&d)[NT][4], const uint32_t (&a)[4], const uint32_t (&b0)[NT],
                          const uint32_t (&b1)[NT], bool fresh) {
  const float z[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    if (fresh) mma_f16(d[t], a, b0[t], b1[t], z);
    else mma_f16(d[t], a, b0[t], b1[t], d[t]);
  }
}
template <int NT>
FP4X_DEV void mma_bf16_acc(float (&d)[NT][4], const uint32_t (&a)[4], const uint32_t (&b0)[NT],
                           const uint32_t (&b1)[NT]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) mma_bf16(d[t], a, b0[t], b1[t], d[t]);
}

// A stage holds NB0 boxes of CPB 16-byte chunks (CPB = 8 for 128-byte boxes, 4 for 64-byte boxes) of 64 rows.
// The two k-groups of consumer warps split it: each processes NCHK consecutive chunks of one box (box b, first
// chunk c0).  The stage functions are fully unrolled over NCHK; every shared-memory load of the range (ldmatrix
// fragments, activation fragments, scales) is issued before the arithmetic that consumes it, and formats that chain
// MMAs spread them over independent accumulators.

template <int NT, int NACC>
FP4X_DEV void zero_accs(float (&a)[NACC][NT][4]) {
#pragma unroll
  for (int i = 0; i < NACC; ++i) zero4<NT>(a[i]);
}
template <int NT, int NACC>
FP4X_DEV void fold_accs(float (&acc)[NT][4], const float (&a)[NACC][NT][4]) {
#pragma unroll
  for (int t = 0; t < NT; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float v = a[0][t][e];
#pragma unroll
      for (int i = 1; i < NACC; ++i) v += a[i][t][e];
      acc[t][e] += v;
    }
}

// NB consecutive scale bytes (NB = 1, 2 or 4; the address is NB-aligned) in the low bytes of a word
template <int NB>
FP4X_DEV uint32_t ld_bytes(uint32_t addr) {
  if (NB == 4) return lds32(addr);
  if (NB == 2) return lds16(addr);
  return lds8(addr);
}

// MXFP8: a chunk pair is one 32-group G; steps 2G + h; group scales applied to the fp32 group sums
template <int NT, int NCHK>
FP4X_DEV void stage_mx8(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  constexpr int NG = NCHK / 2;
  const int G0 = (b * c.CPB + c0) >> 1;
  uint32_t r[NG][4];
  uint32_t b0[2 * NG][NT], b1[2 * NG][NT];
#pragma unroll
  for (int j = 0; j < NG; ++j) ld_pair(c, b, c0 + 2 * j, r[j][0], r[j][1], r[j][2], r[j][3]);
#pragma unroll
  for (int s = 0; s < 2 * NG; ++s) load_b<NT>(c, 2 * G0 + s, b0[s], b1[s]);
  const uint32_t slo = ld_bytes<NG>(c.sc + (c.rbase + c.g) * c.SB + G0);
  const uint32_t shi = ld_bytes<NG>(c.sc + (c.rbase + c.g + 8) * c.SB + G0);
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    float tmp[NT][4];
    const uint32_t A0[4] = {e4m3x2_to_f16x2(r[j][0]), e4m3x2_to_f16x2(r[j][1]), e4m3x2_to_f16x2(r[j][0] >> 16),
                            e4m3x2_to_f16x2(r[j][1] >> 16)};
    mma_f16_acc<NT>(tmp, A0, b0[2 * j], b1[2 * j], true);
    const uint32_t A1[4] = {e4m3x2_to_f16x2(r[j][2]), e4m3x2_to_f16x2(r[j][3]), e4m3x2_to_f16x2(r[j][2] >> 16),
                            e4m3x2_to_f16x2(r[j][3] >> 16)};
    mma_f16_acc<NT>(tmp, A1, b0[2 * j + 1], b1[2 * j + 1], false);
    const float sl = e8m0_to_f32((slo >> (8 * j)) & 0xffu);
    const float sh = e8m0_to_f32((shi >> (8 * j)) & 0xffu);
    fma_scaled<NT>(acc, tmp, sl, sh);
  }
}

// W8 weights exactly as the reference forms them (K:126-130): bf16(f32(q) * s) per weight, s the fp32 group scale.
// A byte b = q + 128 (the code with its sign bit flipped) placed in bits 8..15 of 1.0f gives f = 1 + b * 2^-15;
// f - (1 + 2^-8) = q * 2^-15 exactly, and multiplying by s * 2^15 (exact) rounds once, to fp32(q * s).  The pair
// is then rounded to bf16x2.  `u` holds four biased codes; `h` picks bytes (0, 1) or (2, 3).
FP4X_DEV uint32_t w8_bf16_pair(uint32_t u, int h, uint64_t s2) {
  const uint32_t f0 = prmt(u, 0x3F800000u, h ? 0x7624u : 0x7604u);
  const uint32_t f1 = prmt(u, 0x3F800000u, h ? 0x7634u : 0x7614u);
  const uint64_t kBias = 0xBF808000BF808000ull;  // (-(1 + 2^-8), -(1 + 2^-8))
  return f32x2_to_bf16x2(f32x2_mul(f32x2_add(f32x2_from_bits(f0, f1), kBias), s2));
}

// W8: four chunks per 64-group G; steps 4G + h.  Weights decoded to the reference's bf16 values, bf16 MMAs on the
// raw bf16 activations.
template <int NT, int NCHK>
FP4X_DEV void stage_w8(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  constexpr int NG = NCHK / 4;
  constexpr int NACC = 2;
  const int G0 = (b * c.CPB + c0) >> 2;
  uint32_t r[NG][8];
  uint32_t b0[4 * NG][NT], b1[4 * NG][NT];
  float slo[NG], shi[NG];
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    ld_pair(c, b, c0 + 4 * j, r[j][0], r[j][1], r[j][2], r[j][3]);
    ld_pair(c, b, c0 + 4 * j + 2, r[j][4], r[j][5], r[j][6], r[j][7]);
  }
#pragma unroll
  for (int s = 0; s < 4 * NG; ++s) load_b<NT>(c, 4 * G0 + s, b0[s], b1[s]);
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    slo[j] = __uint_as_float(lds32(c.sc + (c.rbase + c.g) * c.SB + 4 * (G0 + j)));
    shi[j] = __uint_as_float(lds32(c.sc + (c.rbase + c.g + 8) * c.SB + 4 * (G0 + j)));
  }
  float accs[NACC][NT][4];
  zero_accs<NT, NACC>(accs);
#pragma unroll
  for (int j = 0; j < NG; ++j) {
    const uint64_t s2lo = f32x2_splat(slo[j] * 32768.f), s2hi = f32x2_splat(shi[j] * 32768.f);
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const uint32_t lo = r[j][2 * h] ^ 0x80808080u, hi = r[j][2 * h + 1] ^ 0x80808080u;  // rows g, g+8
      const uint32_t A[4] = {w8_bf16_pair(lo, 0, s2lo), w8_bf16_pair(hi, 0, s2hi), w8_bf16_pair(lo, 1, s2lo),
                             w8_bf16_pair(hi, 1, s2hi)};
      mma_bf16_acc<NT>(accs[h % NACC], A, b0[4 * j + h], b1[4 * j + h]);
    }
  }
  fold_accs<NT, NACC>(acc, accs);
}

// Two 6-bit codes of a W6 pair word (code c_lo in bits 0..5, c_hi in bits 16..21 over the constant 0x3F803F80) to
// the reference's bf16((c - 32) * s) (K:160-170).  Each half moved to the top of a word is the fp32 value
// 1 + c * 2^-7; (c - 32) * s = f * (128 s) - 160 s, where 128 s and 160 s are exact (s is an fp16 value) and the
// result has at most 17 significant bits, so one fused multiply-add gives it exactly and the bf16 rounding is the
// reference's single rounding.
FP4X_DEV uint32_t w6_bf16_pair(uint32_t w, uint64_t s128, uint64_t s160n) {
  return f32x2_to_bf16x2(f32x2_fma(f32x2_from_bits(w << 16, w & 0xFFFF0000u), s128, s160n));
}

FP4X_DEV uint32_t w6_lane(uint32_t lo_src, uint32_t hi_src) {
  return (lo_src & 0x000F000Fu) | (hi_src & 0x00300030u) | 0x3F803F80u;
}

// W6: a chunk of the low-nibble plane is one 32-group G (thread: 8 k = 32G + 8tq + r); steps 2G + h.
// W6 stages always use 128-byte low-nibble boxes; NCHK 8 is the two-box stage (512 k: 128-byte high-bit rows,
// 32 scale bytes per row), NCHK 4 the one-box stage (256 k: 64-byte high-bit rows, 16 scale bytes).  Every
// address of the stage is a per-thread base XOR a constant: the bases have the varying bits clear (1024-aligned
// planes, whole rows), and the varying parts (chunk pair, group) sit in bits the thread's fixed parts leave free.
// W6 one-box range: four 32-groups starting at group G0 (low-nibble chunk pair address a0, high-bit and scale row
// bases hb / sb already offset to G0).  All shared-memory loads of the range are issued before its arithmetic.
template <int NT>
FP4X_DEV void w6_groups4(const WarpCtx& c, uint32_t a0, const uint32_t (&hb)[2], const uint32_t (&sb)[2], int G0,
                         float (&accs)[2][NT][4]) {
  uint32_t r[2][4];
  uint32_t hs[4][2];
  uint32_t b0[8][NT], b1[8][NT];
  uint32_t sw[2][2];
#pragma unroll
  for (int u = 0; u < 2; ++u) ldsm_x4(a0 ^ (32u * u), r[u][0], r[u][1], r[u][2], r[u][3]);
#pragma unroll
  for (int gg = 0; gg < 4; ++gg)
#pragma unroll
    for (int q = 0; q < 2; ++q) hs[gg][q] = lds16(hb[q] ^ (8u * gg));
#pragma unroll
  for (int s = 0; s < 8; ++s) load_b<NT>(c, 2 * G0 + s, b0[s], b1[s]);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    sw[0][i] = lds32(sb[0] + 4 * i);
    sw[1][i] = lds32(sb[1] + 4 * i);
  }
#pragma unroll
  for (int gg = 0; gg < 4; ++gg) {
    uint32_t L[2], Hs[2];
    uint64_t s128[2], s160[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      L[q] = r[gg >> 1][2 * (gg & 1) + q];
      Hs[q] = prmt(hs[gg][q], 0u, 0x4140u);
      const float s = f16_bits_to_f32((sw[q][gg >> 1] >> (16 * (gg & 1))) & 0xffffu);
      s128[q] = f32x2_splat(128.f * s);
      s160[q] = f32x2_splat(-160.f * s);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t A[4];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t lo, hi;
        if (h == 0) {
          lo = w6_lane(L[q], Hs[q] << 4);         // elements r0, r4
          hi = w6_lane(L[q] >> 4, Hs[q]);         // r1, r5
        } else {
          lo = w6_lane(L[q] >> 8, Hs[q] << 2);    // r2, r6
          hi = w6_lane(L[q] >> 12, Hs[q] >> 2);   // r3, r7
        }
        A[q] = w6_bf16_pair(lo, s128[q], s160[q]);
        A[2 + q] = w6_bf16_pair(hi, s128[q], s160[q]);
      }
      mma_bf16_acc<NT>(accs[h], A, b0[2 * gg + h], b1[2 * gg + h]);
    }
  }
}

// W6: a chunk of the low-nibble plane is one 32-group G (thread: 8 k = 32G + 8tq + r); steps 2G + h.
// W6 stages always use 128-byte low-nibble boxes; NCHK 8 is the two-box stage (512 k: 128-byte high-bit rows,
// 32 scale bytes per row), NCHK 4 the one-box stage (256 k: 64-byte high-bit rows, 16 scale bytes).  Every
// address of the stage is a per-thread base XOR a constant: the bases have the varying bits clear (1024-aligned
// planes, whole rows), and the varying parts (chunk pair, group) sit in bits the thread's fixed parts leave free.
// The two-box stage runs as two four-group halves, which bounds the registers a warp holds.
template <int NT, int NCHK>
FP4X_DEV void stage_w6(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  constexpr int BI1 = NCHK == 8 ? 128 : 64;
  constexpr int SB = NCHK == 8 ? 32 : 16;
  const int G0 = b * 8 + c0;
  const uint32_t a0 = c.p0 + (uint32_t)b * (uint32_t)(kRB * 128) + c.lrow0 + 16u * (uint32_t)((c0 + c.lsel) ^ c.lswz);
  uint32_t hb[2], sb[2];
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    const int row = c.rbase + c.g + 8 * q;
    hb[q] = c.p1 + swz((uint32_t)(row * BI1 + 8 * G0 + 2 * c.tq), BI1);
    sb[q] = c.sc + (uint32_t)(row * SB + 2 * G0);
  }
  float accs[2][NT][4];
  zero_accs<NT, 2>(accs);
#pragma unroll
  for (int half = 0; half < NCHK / 4; ++half) {
    const uint32_t hbh[2] = {hb[0] ^ (32u * half), hb[1] ^ (32u * half)};
    const uint32_t sbh[2] = {sb[0] + 8u * half, sb[1] + 8u * half};
    w6_groups4<NT>(c, a0 ^ (64u * half), hbh, sbh, G0 + 4 * half, accs);
  }
  fold_accs<NT, 2>(acc, accs);
}

// NVFP4: a chunk C is 32 k = two 16-groups (thread: k = 32C + 8tq + 4h + i, group 2C + tq/2); steps 2C + h.
// The e4m3 block scale multiplies the e2m1 values in f16 (exact: <= 6 significant bits, normal range).
template <int NT, int NCHK>
FP4X_DEV void stage_nv4(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  constexpr int NACC = 4;
  const int C0 = b * c.CPB + c0;
  uint32_t r[NCHK / 2][4];
  uint32_t b0[2 * NCHK][NT], b1[2 * NCHK][NT];
  uint32_t sc8[NCHK][2];
#pragma unroll
  for (int u = 0; u < NCHK / 2; ++u) ld_pair(c, b, c0 + 2 * u, r[u][0], r[u][1], r[u][2], r[u][3]);
#pragma unroll
  for (int s = 0; s < 2 * NCHK; ++s) load_b<NT>(c, 2 * C0 + s, b0[s], b1[s]);
#pragma unroll
  for (int cc = 0; cc < NCHK; ++cc) {
    const int grp = 2 * (C0 + cc) + (c.tq >> 1);
    sc8[cc][0] = lds8(c.sc + (c.rbase + c.g) * c.SB + grp);
    sc8[cc][1] = lds8(c.sc + (c.rbase + c.g + 8) * c.SB + grp);
  }
  float accs[NACC][NT][4];
  zero_accs<NT, NACC>(accs);
#pragma unroll
  for (int cc = 0; cc < NCHK; ++cc) {
    const uint32_t s2lo = prmt(e4m3x2_to_f16x2(sc8[cc][0]), 0u, 0x1010u);
    const uint32_t s2hi = prmt(e4m3x2_to_f16x2(sc8[cc][1]), 0u, 0x1010u);
    const uint32_t wlo = r[cc >> 1][2 * (cc & 1)], whi = r[cc >> 1][2 * (cc & 1) + 1];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t A[4] = {hmul2(e2m1x2_to_f16x2(wlo >> (16 * h)), s2lo),
                             hmul2(e2m1x2_to_f16x2(whi >> (16 * h)), s2hi),
                             hmul2(e2m1x2_to_f16x2(wlo >> (16 * h + 8)), s2lo),
                             hmul2(e2m1x2_to_f16x2(whi >> (16 * h + 8)), s2hi)};
      mma_f16_acc<NT>(accs[(2 * cc + h) % NACC], A, b0[2 * cc + h], b1[2 * cc + h], false);
    }
  }
  fold_accs<NT, NACC>(acc, accs);
}

// BF16: a chunk pair is one standard 16-k step
template <int NT, int NCHK>
FP4X_DEV void stage_bf16(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  constexpr int NS_ = NCHK / 2, NACC = NS_ < 2 ? 1 : 2;
  const int S0 = (b * c.CPB + c0) >> 1;
  uint32_t A[NS_][4];
  uint32_t b0[NS_][NT], b1[NS_][NT];
#pragma unroll
  for (int s = 0; s < NS_; ++s) ld_pair(c, b, c0 + 2 * s, A[s][0], A[s][1], A[s][2], A[s][3]);
#pragma unroll
  for (int s = 0; s < NS_; ++s) load_b<NT>(c, S0 + s, b0[s], b1[s]);
  float accs[NACC][NT][4];
  zero_accs<NT, NACC>(accs);
#pragma unroll
  for (int s = 0; s < NS_; ++s) mma_bf16_acc<NT>(accs[s % NACC], A[s], b0[s], b1[s]);
  fold_accs<NT, NACC>(acc, accs);
}

// INT2 group table: bytes T[c] (c = code) of bf16 values (-a, -b, +b, +a), a = bf16(1.5 s), b = bf16(0.5 s)
FP4X_DEV void int2_table(uint32_t s16, uint32_t& tlo, uint32_t& thi) {
  const float s = f16_bits_to_f32(s16);
  const uint32_t pk = pack_bf16x2(0.5f * s, 1.5f * s);  // bytes [b_lo, b_hi, a_lo, a_hi]
  tlo = prmt(pk, 0u, 0x2002u);
  thi = prmt(pk, 0u, 0x3113u) ^ 0x00008080u;
}

// INT2: a chunk C is 64 k = four 16-groups; thread tq owns group 4C + tq; steps 4C + p.
// Processed in 128-k units (two chunks, eight steps) to bound the registers held.  The four partial sums are folded
// into `acc` after every unit, so a row's summation order within a k-group's chunks depends on K alone and not on
// the grid: vocabulary shards of one head then give bit-identical logits.
template <int NT, int NCHK>
FP4X_DEV void stage_int2(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  constexpr int NACC = 4;
#pragma unroll
  for (int u = 0; u < NCHK / 2; ++u) {
    float accs[NACC][NT][4];
    zero_accs<NT, NACC>(accs);
    uint32_t rr[4];
    ld_pair(c, b, c0 + 2 * u, rr[0], rr[1], rr[2], rr[3]);
    const int C0 = b * c.CPB + c0 + 2 * u;
    uint32_t s16[2][2];
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int sidx = (4 * (C0 + cc) + c.tq) >> c.gshift;
      s16[cc][0] = lds16(c.sc + (c.rbase + c.g) * c.SB + 2 * sidx);
      s16[cc][1] = lds16(c.sc + (c.rbase + c.g + 8) * c.SB + 2 * sidx);
    }
    uint32_t b0[8][NT], b1[8][NT];
#pragma unroll
    for (int s = 0; s < 8; ++s) load_b<NT>(c, 4 * C0 + s, b0[s], b1[s]);
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      uint32_t tlo[2], thi[2];
      int2_table(s16[cc][0], tlo[0], thi[0]);
      int2_table(s16[cc][1], tlo[1], thi[1]);
      const uint32_t W[2] = {rr[2 * cc], rr[2 * cc + 1]};
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint32_t A[4];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t z = (W[q] >> (2 * p)) & 0x03030303u;
          const uint32_t sl = z * 0x11u + 0x4040u;
          const uint32_t sh = __umulhi(z, 0x110000u) + 0x4040u;
          A[q] = prmt(tlo[q], thi[q], sl);
          A[2 + q] = prmt(tlo[q], thi[q], sh);
        }
        mma_bf16_acc<NT>(accs[p], A, b0[4 * cc + p], b1[4 * cc + p]);
      }
    }
    fold_accs<NT, NACC>(acc, accs);
  }
}

template <int FMT, int NT, int NCHK>
FP4X_DEV void stage_range(const WarpCtx& c, int b, int c0, float (&acc)[NT][4]) {
  if constexpr (FMT == FMT_MX8) stage_mx8<NT, NCHK>(c, b, c0, acc);
  else if constexpr (FMT == FMT_W8) stage_w8<NT, NCHK>(c, b, c0, acc);
  else if constexpr (FMT == FMT_W6) stage_w6<NT, NCHK>(c, b, c0, acc);
  else if constexpr (FMT == FMT_NV4) stage_nv4<NT, NCHK>(c, b, c0, acc);
  else if constexpr (FMT == FMT_BF16) stage_bf16<NT, NCHK>(c, b, c0, acc);
  else stage_int2<NT, NCHK>(c, b, c0, acc);
}

// This k-group's half of a stage.  Stage shapes used by the planner: two 128-byte boxes (each k-group takes one
// box), one 128-byte box (four chunks each), one 64-byte box (two chunks each; a W8 64-group spans the whole box, so
// k-group 0 takes it alone).
// The stage shape is a template parameter of the kernel (SHAPE_*), so each kernel holds the code of one shape:
// the fully unrolled stage bodies are large, and a kernel carrying all three shapes runs out of instruction cache.
enum StageShape : int { SHAPE_128x2 = 0, SHAPE_128x1 = 1, SHAPE_64x1 = 2 };

template <int FMT, int NT, int SHAPE>
FP4X_DEV void compute_stage(const WarpCtx& c, int kg, float (&acc)[NT][4]) {
  if constexpr (SHAPE == SHAPE_128x2) {
    stage_range<FMT, NT, 8>(c, kg, 0, acc);
  } else if constexpr (SHAPE == SHAPE_128x1) {
    stage_range<FMT, NT, 4>(c, 0, 4 * kg, acc);
  } else if constexpr (FMT == FMT_W8) {
    if (kg == 0) stage_range<FMT, NT, 4>(c, 0, 0, acc);
  } else {
    stage_range<FMT, NT, 2>(c, 0, 2 * kg, acc);
  }
}

// ------------------------------------------------------------------------------------------------------
// epilogues (values v are this warp's 16 rows: c0,c1 row g; c2,c3 row g+8; columns 8t + 2tq + (0,1))
// ------------------------------------------------------------------------------------------------------
// hyper-connection down epilogue (fused and unfused paths share it): di = bf16(v); bot = bf16(t*sigmoid(t)),
// t = bf16(f32(di) / hc), for columns < lr
FP4X_DEV void hc_down_store(__nv_bfloat16* di, __nv_bfloat16* bot, int N, int lr, int hc, int m, int n, float v) {
  const __nv_bfloat16 d = __float2bfloat16_rn(v);
  di[(int64_t)m * N + n] = d;
  if (n < lr && bot) {
    const float f = __bfloat162float(d);
    const float t = bf16_round(hc == 4 ? f * 0.25f : f / (float)hc);  // / 4 is exact as * 0.25
    bot[(int64_t)m * lr + n] = __float2bfloat16_rn(t * sigmoidf_(t));
  }
}

// gate-mean for one output: out = bf16( ((p0 + p1) + (p2 + p3) ...) / hc ), p_s = bf16(nrm_s * gate_s)
FP4X_DEV float hc_gate_mean(const float* nrm_vals, const float* gates, int hc) {
  float p[8];
  for (int s = 0; s < hc; ++s) p[s] = bf16_round(nrm_vals[s] * gates[s]);
  int n = hc;
  while (n > 1) {
    int w = 0;
    for (int i = 0; i < n; i += 2) p[w++] = (i + 1 < n) ? (p[i] + p[i + 1]) : p[i];
    n = w;
  }
  return bf16_round(p[0] / (float)hc);
}

// HC up: pull the normalized-stream values that the epilogue of row block `blk` reads (the same indices as
// run_epilogue's gate-mean loop, for row warp `wrow`) into L1 while the block's stages stream.  The epilogue runs
// after the reduction, where these loads would otherwise wait a full L2 round trip.
FP4X_DEV void hc_up_prefetch_nrm(const GemvArgs& A, int blk, int wrow, int lane) {
  const int rows = A.hc * A.bj;
  const int first = rows == 32 ? (wrow & ~1) : wrow, nw = rows == 32 ? 2 : 1;
  const int blk_row0 = blk * kRB + 16 * first;
  if (blk_row0 >= A.N) return;
  const int jb = blk_row0 / rows, H = A.N / A.hc;
  const __nv_bfloat16* nrm = reinterpret_cast<const __nv_bfloat16*>(A.nrm);
  const int nout = A.bj * A.M;
  for (int o = lane + 32 * (wrow - first); o < nout; o += 32 * nw) {
    const int m = o / A.bj, col = jb * A.bj + (o - m * A.bj);
    for (int sidx = 0; sidx < A.hc; ++sidx)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(nrm + (int64_t)m * A.nrm_stride + sidx * H + col));
  }
}

template <int EPI, int NT>
FP4X_DEV void run_epilogue(const GemvArgs& A, const GemvItem& it, int row0, const float (&v)[NT][4], int warp, int g,
                           int tq, float* scr_all) {
  constexpr int MP = 8 * NT;
  if (EPI == EPI_STORE || EPI == EPI_HEAD || EPI == EPI_HC_DOWN) {
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int n = row0 + g + 8 * (e >> 1);
        const int m = 8 * t + 2 * tq + (e & 1);
        if (n < A.N && m < A.M) {
          if (EPI == EPI_HC_DOWN) {
            hc_down_store(reinterpret_cast<__nv_bfloat16*>(it.out), reinterpret_cast<__nv_bfloat16*>(it.out2), A.N,
                          A.lr, A.hc, m, n, v[t][e]);
          } else {
            const float val = v[t][e] * A.post;
            store_out(it.out, A.out_dtype, (int64_t)m * A.out_stride + n, val);
            if (EPI == EPI_HEAD && it.out2)
              reinterpret_cast<__nv_bfloat16*>(it.out2)[(int64_t)m * A.out_stride + n] = __float2bfloat16_rn(val);
          }
        }
      }
  } else {  // EPI_HC_UP: interleaved blocks of hc * bj rows (16 rows: one warp; 32 rows: a warp pair)
    float* scr = scr_all + warp * 16 * MP;
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = g + 8 * (e >> 1);
        const int m = 8 * t + 2 * tq + (e & 1);
        scr[r * MP + m] = bf16_round(sigmoidf_(bf16_round(v[t][e])));
      }
    const int rows = A.hc * A.bj;
    const int lane = 4 * g + tq;
    int first_warp = warp, nwarps = 1;
    if (rows == 32) {
      first_warp = warp & ~1;
      nwarps = 2;
      named_bar(2 + (warp >> 1), 64);
    } else {
      __syncwarp();
    }
    const float* bscr = scr_all + first_warp * 16 * MP;  // the block's rows, contiguous over the warp pair
    const int blk_row0 = row0 - 16 * (warp - first_warp);
    if (blk_row0 < A.N) {
      const int jb = blk_row0 / rows;  // interleave block index
      const int H = A.N / A.hc;
      const __nv_bfloat16* nrm = reinterpret_cast<const __nv_bfloat16*>(A.nrm);
      const int nout = A.bj * A.M;
      if (A.hc == 4) {
        // four streams (the served and benchmarked geometry): the loads of an output issue together and the
        // values stay in registers; the same products and the same pairwise sum order as hc_gate_mean, and
        // the division by 4 is exact as a multiplication
        for (int o = lane + 32 * (warp - first_warp); o < nout; o += 32 * nwarps) {
          const int m = o / A.bj, cidx = o - m * A.bj;
          const int col = jb * A.bj + cidx;
          const __nv_bfloat16* nr = nrm + (int64_t)m * A.nrm_stride + col;
          float p[4];
#pragma unroll
          for (int s4 = 0; s4 < 4; ++s4)
            p[s4] = bf16_round(__bfloat162float(nr[s4 * H]) * bscr[(s4 * A.bj + cidx) * MP + m]);
          reinterpret_cast<__nv_bfloat16*>(it.out)[(int64_t)m * A.out_stride + col] =
              __float2bfloat16_rn(bf16_round(((p[0] + p[1]) + (p[2] + p[3])) * 0.25f));
        }
      } else
      for (int o = lane + 32 * (warp - first_warp); o < nout; o += 32 * nwarps) {
        const int m = o / A.bj, cidx = o - m * A.bj;
        const int col = jb * A.bj + cidx;
        float nv[8], gv[8];
        for (int s = 0; s < A.hc; ++s) {
          nv[s] = __bfloat162float(nrm[(int64_t)m * A.nrm_stride + s * H + col]);
          gv[s] = bscr[(s * A.bj + cidx) * MP + m];
        }
        reinterpret_cast<__nv_bfloat16*>(it.out)[(int64_t)m * A.out_stride + col] =
            __float2bfloat16_rn(hc_gate_mean(nv, gv, A.hc));
      }
    }
    if (rows == 32) named_bar(2 + (warp >> 1), 64);
    else __syncwarp();
  }
}

// ------------------------------------------------------------------------------------------------------
// the kernel
// ------------------------------------------------------------------------------------------------------
template <int FMT, int NT, int EPI, int SHAPE>
FP4X_DEV void gemv_body(const GemvArgs& A) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // stages need 1024-byte alignment for the swizzled TMA tiles; the host adds 1 KB of slack
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  constexpr int MP = 8 * NT;
  constexpr FmtGeom G = fmt_geom(FMT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = blockIdx.y, b = blockIdx.z;
  const int k_panel0 = p * A.KPW;
  GemvItem it = A.item;
  const CUtensorMap* tm0 = &A.tm0;
  if (A.batch) {
    const BatchEntry* e = A.batch + b;
    tm0 = &e->tm0;
    it.x = e->x;
    it.sc = e->sc;
    it.out = e->out;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + A.smem_misc + 128);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kMaxStages);
  const uint32_t xbar = smem_u32(bars + 2 * kMaxStages);
  // k-group handshake per row warp: comb_full (k-group 1 has left its sums), comb_empty (k-group 0 has read them)
  const uint32_t comb_full0 = smem_u32(bars + 2 * kMaxStages + 1), comb_empty0 = comb_full0 + 8 * kRW;
  // cluster leader: one barrier per row warp that the other panels' CTAs arrive on remotely
  const uint32_t red_full0 = comb_empty0 + 8 * kRW;
  const int CPP = A.CPP;
  const int cta = blockIdx.x;
  const int64_t Up = A.whole ? (int64_t)A.RT : (int64_t)A.RT * A.NCH;
  const int64_t u_begin = A.whole ? range_begin(A.RT, CPP, cta) * A.NCH : range_begin(Up, CPP, cta);
  const int64_t u_end = A.whole ? range_begin(A.RT, CPP, cta + 1) * A.NCH : range_begin(Up, CPP, cta + 1);
  const int64_t nunits = u_end - u_begin;

  if (threadIdx.x == 0) {
    FP4X_TL(tl_first(A.tl, kTlStartFirst); tl_last(A.tl, kTlStartLast));  // timeline: CTA start
    for (int s = 0; s < A.NS; ++s) {
      mbar_init(full0 + 8 * s, 33);
      mbar_init(empty0 + 8 * s, kCWarps);
    }
    mbar_init(xbar, 1);
    for (int i = 0; i < kRW; ++i) {
      mbar_init(comb_full0 + 8 * i, 1);
      mbar_init(comb_empty0 + 8 * i, 1);
      if (A.cluster > 1) {
        // the leader arrives here once, expecting the other panels' partial sums as bytes (st.async complete_tx),
        // before the cluster barrier below lets any of them store
        mbar_init(red_full0 + 8 * i, 1);
        if (cluster_ctarank() == 0)
          mbar_arrive_expect_tx(red_full0 + 8 * i, (uint32_t)(A.cluster - 1) * 32u * NT * 16u);
      }
    }
    mbar_init_fence();
  }
  __syncthreads();
  // the leader's barriers must be initialised before another CTA of the cluster arrives on them
  if (A.cluster > 1) cluster_sync_all();

  if (warp == kCWarps) {
    // ---------------- producer warp ----------------
    pdl_launch_dependents();
    const int tx = kRB * (A.NB0 * A.BI0 + (G.n1 ? A.BI1 : 0));
    const int scw = A.scw;
    const int words_per_row = G.sn ? A.SB / scw : 0;
    const int sd = FMT == FMT_INT2 ? A.group / 2 : G.sd;
    int s = 0, round = 0;
    int blk = (int)(u_begin / A.NCH), chunk = (int)(u_begin - (int64_t)blk * A.NCH);
    for (int64_t q = 0; q < nunits; ++q) {
      if (round > 0) {
        if (!mbar_wait_bounded(empty0 + 8 * s, (uint32_t)((round - 1) & 1), A.err)) break;
      }
      const int k0 = k_panel0 + chunk * A.KC;
      const uint32_t stage = smem_u32(base) + (uint32_t)s * A.STG;
      const uint32_t bar = full0 + 8 * s;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar, (uint32_t)tx);
        const int xb0 = k0 * G.n0 / G.d0;
        for (int bx = 0; bx < A.NB0; ++bx)
          tma_load_2d(stage + bx * kRB * A.BI0, tm0, xb0 + bx * A.BI0, blk * kRB, bar);
        if constexpr (G.n1 != 0) tma_load_2d(stage + A.off_p1, &A.tm1, k0 * G.n1 / G.d1, blk * kRB, bar);
      }
      if constexpr (G.sn != 0) {
        const int64_t koff = (int64_t)k0 * G.sn / sd;
        const uint32_t sbase = stage + A.off_sc;
        for (int w = lane; w < kRB * words_per_row; w += 32) {
          const int r = w / words_per_row, cw = w - r * words_per_row;
          const int row = min(blk * kRB + r, A.N - 1);
          const uint8_t* src = it.sc + (int64_t)row * A.lds + koff + (int64_t)cw * scw;
          const uint32_t dst = sbase + r * A.SB + cw * scw;
          if (scw == 16) cp_async16(dst, src);
          else if (scw == 8) cp_async8(dst, src);
          else cp_async4(dst, src);
        }
      }
      cp_async_arrive_noinc(bar);
      if (++s == A.NS) { s = 0; ++round; }
      if (++chunk == A.NCH) { chunk = 0; ++blk; }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    return;
  }

  // ---------------- consumer warps ----------------
  // start of this CTA's work: a cluster non-leader writes into the leader's shared memory only within 1 s of it, and
  // the leader waits 2 s from a later moment (its own wait), so no remote write can land after the leader gave up
  // (the CTAs of a cluster start together)
  const uint64_t t_start = A.cluster > 1 ? global_ns() : 0;
  const int g = lane >> 2, tq = lane & 3;
  const int wrow = warp & (kRW - 1), kg = warp / kRW;
  pdl_wait();
  FP4X_TL(if (threadIdx.x == 0) { tl_last(A.tl, kTlWaitLast); tl_first(A.tl, kTlWaitFirst); });
  stage_activations<FMT, NT>(A, it, base, MP, k_panel0, xbar);
  named_bar(1, kCWarps * 32);
  pdl_launch_dependents();
  FP4X_TL(if (threadIdx.x == 0) tl_last(A.tl, kTlStaged));

  const float* xsc = reinterpret_cast<const float*>(base + A.smem_misc);
  float* scr = reinterpret_cast<float*>(base + A.smem_scr);
  WarpCtx wc;
  wc.BI0 = A.BI0; wc.BI1 = A.BI1; wc.NB0 = A.NB0; wc.SB = A.SB; wc.XP = A.XP; wc.CPB = A.BI0 / 16;
  wc.g = g; wc.tq = tq; wc.rbase = 16 * wrow;
  wc.gshift = A.group == 32 ? 1 : 0;
  {
    const int r = 16 * wrow + (lane & 7) + 8 * ((lane >> 3) & 1);
    wc.lrow0 = (uint32_t)(r * A.BI0);
    wc.lswz = A.BI0 == 128 ? (r & 7) : ((r >> 1) & 3);
    wc.lsel = lane >> 4;
  }
  const uint32_t xrow = smem_u32(base + A.smem_x) + g * A.XP + tq * 8;
  const int steps_per_stage = A.KC / 16;

  float acc[NT][4];
  zero4<NT>(acc);
  int cur = -1;
  bool ok = true;
  uint32_t nflush = 0;
  float* comb = reinterpret_cast<float*>(base + A.smem_comb) + (wrow * 32 + lane) * (NT * 4);

  auto flush = [&](int blk) {
    // k-group 1 hands its partial sums for these 16 rows to k-group 0 through shared memory
    const uint32_t cf_bar = comb_full0 + 8 * wrow, ce_bar = comb_empty0 + 8 * wrow;
    const uint32_t par = nflush & 1u;
    ++nflush;
    if (kg == 1) {
      // the previous block's sums must have been read before this block's overwrite them
      if (nflush > 1 && !mbar_wait_bounded(ce_bar, par ^ 1u, A.err)) { ok = false; return; }
#pragma unroll
      for (int t = 0; t < NT; ++t)
        *reinterpret_cast<float4*>(comb + 4 * t) = make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
      __syncwarp();
      if (lane == 0) mbar_arrive(cf_bar);
      return;
    }
    if (!mbar_wait_bounded(cf_bar, par, A.err)) { ok = false; return; }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const float4 o = *reinterpret_cast<const float4*>(comb + 4 * t);
      acc[t][0] += o.x; acc[t][1] += o.y; acc[t][2] += o.z; acc[t][3] += o.w;
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(ce_bar);
    FP4X_TL(if (lane == 0) tl_last(A.tl, kTlHandover));
    if (G.xf16) {
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[t][e] *= xsc[MP + 8 * t + 2 * tq + (e & 1)];
    }
    const int row0 = blk * kRB + 16 * wrow;
    if (A.cluster > 1) {
      // One row block per CTA; the CTAs of the block's K panels form the cluster.  Each non-leader stores its
      // partial sums into the leader's shared memory with st.async, whose bytes complete the leader's barrier for
      // this row warp; the leader adds them in panel order and runs the epilogue.
      const uint32_t rank = cluster_ctarank();
      constexpr uint32_t kSlot = 32u * NT * 16u;  // one row warp: 32 lanes x NT float4
      const uint32_t red = smem_u32(base + A.smem_red) + (uint32_t)wrow * kSlot + (uint32_t)lane * NT * 16u;
      if (rank != 0) {
        int late = lane == 0 ? (global_ns() - t_start > 1000000000ull) : 0;  // one decision for the warp
        late = __shfl_sync(0xffffffffu, late, 0);
        if (late) {  // too late: the leader may have stopped waiting
          if (lane == 0) set_dev_error(A.err, kDevWaitTimeout);
          ok = false;
          return;
        }
        const uint32_t dst = mapa_shared(red + (rank - 1) * kRW * kSlot, 0);
        // asynchronous remote stores that complete their bytes on the leader's barrier: no release fence and no
        // arrival (measured against st.shared::cluster + a release arrive: 0.1-0.4 µs less per launch)
        const uint32_t rbar = mapa_shared(red_full0 + 8 * wrow, 0);
#pragma unroll
        for (int t = 0; t < NT; ++t) st_async_v4(dst + 16u * t, acc[t][0], acc[t][1], acc[t][2], acc[t][3], rbar);
        return;
      }
      if (!mbar_wait_bounded_cluster(red_full0 + 8 * wrow, 0, A.err)) { ok = false; return; }
      float tot[NT][4];
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) tot[t][e] = acc[t][e];
      for (int r = 1; r < A.cluster; ++r) {
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4 v = *reinterpret_cast<const float4*>(base + A.smem_red + (r - 1) * kRW * kSlot +
                                                            wrow * kSlot + lane * NT * 16 + 16 * t);
          tot[t][0] += v.x; tot[t][1] += v.y; tot[t][2] += v.z; tot[t][3] += v.w;
        }
      }
      FP4X_TL(if (lane == 0) tl_last(A.tl, kTlReduced));
      run_epilogue<EPI, NT>(A, it, row0, tot, wrow, g, tq, scr);
      return;
    }
    int cf, cl;
    if (A.whole) {
      cf = cl = cta;
    } else {
      const int64_t uf = (int64_t)blk * A.NCH, ul = uf + A.NCH - 1;
      cf = owner_of(uf, Up, CPP);
      cl = owner_of(ul, Up, CPP);
    }
    const int segs = cl - cf + 1;
    if (A.KP == 1 && segs == 1) {
      FP4X_TL(if (lane == 0) tl_last(A.tl, kTlReduced));
      run_epilogue<EPI, NT>(A, it, row0, acc, wrow, g, tq, scr);
      return;
    }
    auto slot_of = [&](int pp, int cc) -> int64_t {
      int64_t s;
      if (A.KP == 1) {  // a CTA shares at most two blocks: its first (slot 0) and its last (slot 1)
        const int first_blk = (int)(range_begin(Up, CPP, cc) / A.NCH);
        s = ((int64_t)b * CPP + cc) * 2 + (blk == first_blk ? 0 : 1);
      } else {
        s = (((int64_t)b * A.KP + pp) * A.RT + blk) * A.SMAX + (cc - cf);
      }
      return s * kRW + wrow;
    };
    float* mine = A.ws + slot_of(p, cta) * (16 * MP);
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const int m = 8 * t + 2 * tq;
      __stcg(reinterpret_cast<float2*>(mine + g * MP + m), make_float2(acc[t][0], acc[t][1]));
      __stcg(reinterpret_cast<float2*>(mine + (g + 8) * MP + m), make_float2(acc[t][2], acc[t][3]));
    }
    // The warp barrier orders every lane's partial stores before lane 0's release; the acquire half of the same
    // atomic, followed by the warp barrier, orders the last arriver's reads of the other partials after it.
    __syncwarp();
    int* semp = A.sem + ((int64_t)b * A.RT + blk) * kRW + wrow;
    int last = 0;
    if (lane == 0) last = (atomic_add_acq_rel(semp, 1) == A.KP * segs - 1);
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    if (!last) return;
    // Sum the partial slots in the fixed order (panel, then CTA).  The loads of eight slots are issued before any
    // of them is added (four at M > 8), so their L2 latencies overlap instead of adding up.
    float tot[NT][4];
    zero4<NT>(tot);
    const int nslots = A.KP * segs;
    constexpr int kBatch = 8 / NT;
    for (int i0 = 0; i0 < nslots; i0 += kBatch) {
      float2 v[kBatch][NT][2];
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        const int i = i0 + j;
        if (i < nslots) {
          const int pp = i / segs, cc = cf + (i - pp * segs);
          const float* src = A.ws + slot_of(pp, cc) * (16 * MP);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const int m = 8 * t + 2 * tq;
            v[j][t][0] = __ldcg(reinterpret_cast<const float2*>(src + g * MP + m));
            v[j][t][1] = __ldcg(reinterpret_cast<const float2*>(src + (g + 8) * MP + m));
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kBatch; ++j) {
        if (i0 + j < nslots) {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            tot[t][0] += v[j][t][0].x; tot[t][1] += v[j][t][0].y;
            tot[t][2] += v[j][t][1].x; tot[t][3] += v[j][t][1].y;
          }
        }
      }
    }
    FP4X_TL(if (lane == 0) tl_last(A.tl, kTlReduced));
    run_epilogue<EPI, NT>(A, it, row0, tot, wrow, g, tq, scr);
    if (lane == 0) atomicExch(semp, 0);
  };

  // timeline: first weight stage resident (a wait on phase 0 of stage 0 consumes nothing; only while recording)
  FP4X_TL(if (A.tl && threadIdx.x == 0 && nunits > 0 && mbar_wait_bounded(full0, 0, A.err))
              tl_last(A.tl, kTlFirstStage));
  int s = 0;
  uint32_t phase = 0;
  int blk = (int)(u_begin / A.NCH), chunk = (int)(u_begin - (int64_t)blk * A.NCH);
  for (int64_t q = 0; q < nunits; ++q) {
    if (blk != cur) {
      if (cur >= 0) flush(cur);
      zero4<NT>(acc);
      cur = blk;
      if constexpr (EPI == EPI_HC_UP) {
        if (kg == 0) hc_up_prefetch_nrm(A, blk, wrow, lane);
      }
    }
    if (!mbar_wait_bounded(full0 + 8 * s, phase, A.err)) { ok = false; break; }
    const uint32_t stage = smem_u32(base) + (uint32_t)s * A.STG;
    wc.p0 = stage;
    wc.p1 = stage + A.off_p1;
    wc.sc = stage + A.off_sc;
    wc.xb = xrow + chunk * steps_per_stage * 32;
    compute_stage<FMT, NT, SHAPE>(wc, kg, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
    if (++s == A.NS) { s = 0; phase ^= 1u; }
    if (++chunk == A.NCH) { chunk = 0; ++blk; }
  }
  FP4X_TL(if (threadIdx.x == 0) tl_last(A.tl, kTlLoopDone));
  if (ok && cur >= 0) flush(cur);
  FP4X_TL(if (lane == 0) tl_last(A.tl, kTlStored));
}

// Two entry points with one body.  Plans with more CTAs than SMs keep two CTAs per SM (at most ~100 registers per
// thread); plans with at most one CTA per SM take the wide entry, whose 128-register budget buys the decode loops
// more instruction-level parallelism and still leaves room on the SM for one CTA of the next kernel in the chain.
template <int FMT, int NT, int EPI, int SHAPE>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const __grid_constant__ GemvArgs A) {
  gemv_body<FMT, NT, EPI, SHAPE>(A);
}
template <int FMT, int NT, int EPI, int SHAPE>
__global__ void __maxnreg__(128) gemv_kernel_wide(const __grid_constant__ GemvArgs A) {
  gemv_body<FMT, NT, EPI, SHAPE>(A);
}

}  // namespace fp4x
