// Decode-shaped (M <= 16) quantized GEMV core for sm_100a.
//
//   out[m, n] = sum_k x[m, k] * W[n, k]      x: bf16 [M, K];  W: packed rows in one of six formats
//
// Structure (one CTA per SM, 8 warps):
//   * Work = (row tile of RU = 16*RG rows) x (k chunk of KC elements) "chunk units".  The K axis is cut into KP
//     panels (grid.y); inside a panel the RT*NCH chunk units are split evenly across all CPP*8 warps of the
//     panel (stream-K), so every warp streams the same number of bytes.
//   * Each warp owns a ring of NS shared-memory stages.  Lanes issue one cp.async.bulk per weight row segment
//     (codes) plus 4-byte cp.async for the scale words; an mbarrier per stage completes on the transaction
//     bytes and the 32 async arrivals.  The first NS stages are issued before griddepcontrol.wait (weights
//     never depend on the previous kernel).
//   * The panel's activations are staged once per CTA in shared memory, already permuted into the mma B
//     fragment order of the format and converted to f16 with a per-(token, panel) power-of-two scale (exact for
//     every element within 2^31 of the token's panel maximum) or kept as bf16.
//   * Weights are decoded in registers straight into m16n8k16 A fragments with exact conversions
//     (fp8/fp4 -> f16 cvt, int8/int6 -> f16 magic-number adds, INT2 -> bf16 via a per-group byte-permute table)
//     and multiplied on the tensor cores with fp32 accumulation.  Per-group scales are applied to the fp32
//     group partials (deferred), so products stay exact.
//   * A row tile split across warps or panels is combined by the last arriving warp, which sums the partial
//     slots in a fixed order (deterministic) and runs the epilogue; the arrival counter is reset to zero.
#pragma once
#include "fp4x_common.cuh"

namespace fp4x {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxStages = 8;

enum Fmt : int { FMT_MX8 = 0, FMT_W8 = 1, FMT_W6 = 2, FMT_NV4 = 3, FMT_BF16 = 4, FMT_INT2 = 5 };
enum Epi : int { EPI_STORE = 0, EPI_HC_DOWN = 1, EPI_HC_UP = 2, EPI_HEAD = 3 };

// per-format geometry; bytes-per-k values are num/den
struct FmtGeom {
  int blk;        // k per decode block
  int n0, d0;     // plane-0 bytes per k
  int n1, d1;     // plane-1 bytes per k (0 if absent)
  int sn, sd;     // scale bytes per k (INT2: sd = group / 2)
  int qb;         // activation staging block (consecutive k)
  int xf16;       // activations converted to scaled f16 (else kept bf16)
  int mod0, mod1; // shared-memory pitch residues mod 128 (bank-conflict-free reads)
};

__host__ __device__ constexpr FmtGeom fmt_geom(int fmt) {
  return fmt == FMT_MX8    ? FmtGeom{32, 1, 1, 0, 1, 1, 32, 4, 1, 32, 0}
         : fmt == FMT_W8   ? FmtGeom{64, 1, 1, 0, 1, 1, 16, 4, 1, 64, 0}
         : fmt == FMT_W6   ? FmtGeom{32, 1, 2, 1, 4, 1, 16, 8, 1, 16, 16}
         : fmt == FMT_NV4  ? FmtGeom{128, 1, 2, 0, 1, 1, 16, 4, 1, 64, 0}
         : fmt == FMT_BF16 ? FmtGeom{32, 2, 1, 0, 1, 0, 1, 4, 0, 64, 0}
                           : FmtGeom{256, 1, 4, 0, 1, 1, 8, 16, 0, 64, 0};  // INT2 (scale sd set at runtime)
}

struct GemvItem {
  const void* x;        // bf16 [M, K] (row stride x_stride elements)
  const uint8_t* p0;    // code plane 0
  const uint8_t* p1;    // code plane 1 (W6 high bits)
  const uint8_t* sc;    // scales
  void* out;            // primary output
  void* out2;           // HC down: bottleneck output; head: bf16 copy of the logits
};

struct GemvArgs {
  GemvItem item;          // the matrix of a single call
  const void* const* items4;  // batched W8: device array of {x, codes, scales, out} per grid.z, or null
  int M, N, K;
  int64_t x_stride;
  int64_t ld0, ld1, lds;  // row strides (bytes)
  int64_t out_stride;     // elements between tokens of out (and out2 for the head)
  int out_dtype;
  float post;             // multiplier on the final sum (NVFP4 global scale)
  int KPW, KP;            // panel width and count
  int KC, NCH;            // chunk width and chunks per (row tile, panel)
  int CPP;                // CTAs per (panel, batch item)
  int RT;                 // row tiles
  int NS;                 // stages per warp
  int SMAX;               // partial slots per (batch, panel, row tile) when KP > 1
  int whole;              // 1: warps own whole row tiles (all NCH chunks); no cross-warp reduction
  int group;              // INT2 scale group (16 or 32)
  int P0, P1, PS, STG;    // stage pitches and stage bytes
  int XP;                 // activation token pitch (bytes)
  int smem_x, smem_stage, smem_scr;  // byte offsets of the shared-memory regions
  int lr, hc, bj;         // hyper-connection epilogues
  const void* nrm;        // HC up: normalized input [M, hc*H]
  int64_t nrm_stride;
  float* ws;              // partial slots
  int* sem;               // arrival counters [batch * RT], zero on entry and on exit
  int* err;               // device error word
};

// ------------------------------------------------------------------------------------------------------
// work partition helpers (identical on host and device)
// ------------------------------------------------------------------------------------------------------
__host__ __device__ inline int64_t range_begin(int64_t U, int W, int w) { return U * w / W; }
// warp that owns chunk unit u when U units are split over W warps by range_begin
__host__ __device__ inline int owner_of(int64_t u, int64_t U, int W) { return (int)(((u + 1) * W + U - 1) / U) - 1; }

// ------------------------------------------------------------------------------------------------------
// activation staging: permuted B-fragment order, one quad (4 k values) per (token, step, tq)
// ------------------------------------------------------------------------------------------------------
template <int FMT>
FP4X_DEV void stage_block_positions(int kb, int (&s)[4], int& tq) {
  if (FMT == FMT_MX8 || FMT == FMT_BF16) {  // k0 = 32j + 8tq + 4h
    s[0] = 2 * (kb >> 3) + (kb & 1);
    tq = (kb >> 1) & 3;
  } else if (FMT == FMT_W8) {  // k0 = 64j + 16tq + 4h
    s[0] = 4 * (kb >> 4) + (kb & 3);
    tq = (kb >> 2) & 3;
  } else if (FMT == FMT_NV4) {  // k0 = 128b + 32tq + 4i
    s[0] = 8 * (kb >> 5) + (kb & 7);
    tq = (kb >> 3) & 3;
  } else if (FMT == FMT_W6) {  // k0 = 32j + 8tq, two quads
    s[0] = 2 * (kb >> 2);
    s[1] = s[0] + 1;
    tq = kb & 3;
  } else {  // INT2: k0 = 256b + 64tq + 16gi, four quads
    const int base = 16 * (kb >> 4) + 4 * (kb & 3);
    s[0] = base;
    s[1] = base + 1;
    s[2] = base + 2;
    s[3] = base + 3;
    tq = (kb >> 2) & 3;
  }
}

FP4X_DEV uint32_t cvt_pair(uint32_t bf2, float scl, bool xf16) {
  if (!xf16) return bf2;
  const float lo = bf16_bits_to_f32(bf2 & 0xffffu) * scl;
  const float hi = bf16_bits_to_f32(bf2 >> 16) * scl;
  return pack_f16x2(lo, hi);
}
FP4X_DEV uint32_t pick2(uint32_t lo_src, int lo_idx, uint32_t hi_src, int hi_idx) {
  // gather two 16-bit values (selected halves of two words) into one word
  const uint32_t a = (lo_src >> (16 * lo_idx)) & 0xffffu;
  const uint32_t b = (hi_src >> (16 * hi_idx)) & 0xffffu;
  return a | (b << 16);
}

template <int FMT>
FP4X_DEV void stage_activations(const GemvArgs& A, const GemvItem& it, uint8_t* smem, int MP, int k_panel0) {
  constexpr FmtGeom G = fmt_geom(FMT);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float* xsc = reinterpret_cast<float*>(smem + kWarps * kMaxStages * 8);  // [MP] scale, [MP] inverse
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(it.x);
  const int KPW = A.KPW;
  if (G.xf16) {
    for (int tok = warp; tok < MP; tok += kWarps) {
      float mx = 0.f;
      if (tok < A.M) {
        const uint4* row = reinterpret_cast<const uint4*>(x + (int64_t)tok * A.x_stride + k_panel0);
        for (int i = lane; i < KPW / 8; i += 32) {
          uint4 v = __ldg(row + i);
          uint32_t w[4] = {v.x, v.y, v.z, v.w};
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
    __syncthreads();
  }
  const uint32_t xbase = smem_u32(smem + A.smem_x);
  const int nblk = KPW / G.qb;
  for (int idx = tid; idx < MP * nblk; idx += kThreads) {
    const int tok = idx / nblk, kb = idx - tok * nblk;
    const float scl = G.xf16 ? xsc[tok] : 1.f;
    uint32_t v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (tok < A.M) {
      const __nv_bfloat16* src = x + (int64_t)tok * A.x_stride + k_panel0 + kb * G.qb;
      if (G.qb == 4) {
        uint2 t = *reinterpret_cast<const uint2*>(src);
        v[0] = t.x; v[1] = t.y;
      } else if (G.qb == 8) {
        uint4 t = *reinterpret_cast<const uint4*>(src);
        v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
      } else {
        uint4 t0 = *reinterpret_cast<const uint4*>(src);
        uint4 t1 = *reinterpret_cast<const uint4*>(src + 8);
        v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w;
        v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
      }
    }
    int s[4];
    int tq;
    stage_block_positions<FMT>(kb, s, tq);
    const uint32_t trow = xbase + tok * A.XP + tq * 8;
    if (G.qb == 4) {
      sts64(trow + s[0] * 32, cvt_pair(v[0], scl, G.xf16), cvt_pair(v[1], scl, G.xf16));
    } else if (G.qb == 8) {
      // elements r0..r7 in v[0..3] (two per word); quads (r0,r4,r1,r5) and (r2,r6,r3,r7)
      sts64(trow + s[0] * 32, cvt_pair(pick2(v[0], 0, v[2], 0), scl, G.xf16),
            cvt_pair(pick2(v[0], 1, v[2], 1), scl, G.xf16));
      sts64(trow + s[1] * 32, cvt_pair(pick2(v[1], 0, v[3], 0), scl, G.xf16),
            cvt_pair(pick2(v[1], 1, v[3], 1), scl, G.xf16));
    } else {
      // elements e0..e15 in v[0..7]; quad p = (ORDER[p], 4+ORDER[p], 8+ORDER[p], 12+ORDER[p]), ORDER=(0,2,1,3)
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int o = (p == 1) ? 2 : (p == 2 ? 1 : p);
        // element e lives in v[e/2], half e%2
        const int e0 = o, e1 = 4 + o, e2 = 8 + o, e3 = 12 + o;
        const uint32_t lo = pick2(v[e0 >> 1], e0 & 1, v[e1 >> 1], e1 & 1);
        const uint32_t hi = pick2(v[e2 >> 1], e2 & 1, v[e3 >> 1], e3 & 1);
        sts64(trow + s[p] * 32, cvt_pair(lo, scl, G.xf16), cvt_pair(hi, scl, G.xf16));
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------------
// per-format chunk compute: accumulate one (RU rows x KC) chunk into acc
// ------------------------------------------------------------------------------------------------------
struct ChunkCtx {
  uint32_t a0, a1, sc;  // shared addresses of the stage planes and scales
  int P0, P1, PS;
  int KC;
  uint32_t xb;          // shared address of the activation tile for step 0 of this chunk, token row g, tq
  int XP;
  int g, tq;
  int group;            // INT2 scale group
};

template <int NT>
FP4X_DEV void load_b(const ChunkCtx& c, int s, uint32_t (&b0)[NT], uint32_t (&b1)[NT]) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    uint2 v = lds64(c.xb + t * 8 * c.XP + s * 32);
    b0[t] = v.x;
    b1[t] = v.y;
  }
}

template <int NT, int RG>
FP4X_DEV void zero_acc(float (&a)[RG][NT][4]) {
#pragma unroll
  for (int r = 0; r < RG; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t)
#pragma unroll
      for (int e = 0; e < 4; ++e) a[r][t][e] = 0.f;
}

template <int NT, int RG>
FP4X_DEV void fma_scaled(float (&acc)[RG][NT][4], const float (&tmp)[RG][NT][4], const float (&s_lo)[RG],
                         const float (&s_hi)[RG]) {
#pragma unroll
  for (int r = 0; r < RG; ++r)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      acc[r][t][0] = fmaf(tmp[r][t][0], s_lo[r], acc[r][t][0]);
      acc[r][t][1] = fmaf(tmp[r][t][1], s_lo[r], acc[r][t][1]);
      acc[r][t][2] = fmaf(tmp[r][t][2], s_hi[r], acc[r][t][2]);
      acc[r][t][3] = fmaf(tmp[r][t][3], s_hi[r], acc[r][t][3]);
    }
}

template <int NT, int RG>
FP4X_DEV void chunk_mx8(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = 0; j < c.KC / 32; ++j) {
    uint2 a[RG][2];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int row = 16 * r + c.g;
      a[r][0] = lds64(c.a0 + row * c.P0 + 32 * j + 8 * c.tq);
      a[r][1] = lds64(c.a0 + (row + 8) * c.P0 + 32 * j + 8 * c.tq);
    }
    float tmp[RG][NT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t b0[NT], b1[NT];
      load_b<NT>(c, 2 * j + h, b0, b1);
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const uint32_t w0 = h ? a[r][0].y : a[r][0].x;
        const uint32_t w1 = h ? a[r][1].y : a[r][1].x;
        const uint32_t A[4] = {e4m3x2_to_f16x2(w0), e4m3x2_to_f16x2(w1), e4m3x2_to_f16x2(w0 >> 16),
                               e4m3x2_to_f16x2(w1 >> 16)};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (h == 0)
            mma_f16(tmp[r][t], A, b0[t], b1[t], zero);
          else
            mma_f16(tmp[r][t], A, b0[t], b1[t], tmp[r][t]);
        }
      }
    }
    float sl[RG], sh[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int row = 16 * r + c.g;
      sl[r] = e8m0_to_f32(lds8(c.sc + row * c.PS + j));
      sh[r] = e8m0_to_f32(lds8(c.sc + (row + 8) * c.PS + j));
    }
    fma_scaled<NT, RG>(acc, tmp, sl, sh);
  }
}

template <int NT, int RG>
FP4X_DEV void chunk_w8(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t kMagic = 0x64646464u, kNeg1152 = 0xE480E480u;
  for (int j = 0; j < c.KC / 64; ++j) {
    uint4 a[RG][2];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int row = 16 * r + c.g;
      a[r][0] = lds128(c.a0 + row * c.P0 + 64 * j + 16 * c.tq);
      a[r][1] = lds128(c.a0 + (row + 8) * c.P0 + 64 * j + 16 * c.tq);
    }
    float tmp[RG][NT][4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      uint32_t b0[NT], b1[NT];
      load_b<NT>(c, 4 * j + h, b0, b1);
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const uint32_t w0 = (h == 0 ? a[r][0].x : h == 1 ? a[r][0].y : h == 2 ? a[r][0].z : a[r][0].w) ^ 0x80808080u;
        const uint32_t w1 = (h == 0 ? a[r][1].x : h == 1 ? a[r][1].y : h == 2 ? a[r][1].z : a[r][1].w) ^ 0x80808080u;
        const uint32_t A[4] = {hadd2(prmt(w0, kMagic, 0x4140u), kNeg1152), hadd2(prmt(w1, kMagic, 0x4140u), kNeg1152),
                               hadd2(prmt(w0, kMagic, 0x4342u), kNeg1152), hadd2(prmt(w1, kMagic, 0x4342u), kNeg1152)};
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (h == 0)
            mma_f16(tmp[r][t], A, b0[t], b1[t], zero);
          else
            mma_f16(tmp[r][t], A, b0[t], b1[t], tmp[r][t]);
        }
      }
    }
    float sl[RG], sh[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int row = 16 * r + c.g;
      sl[r] = __uint_as_float(lds32(c.sc + row * c.PS + 4 * j));
      sh[r] = __uint_as_float(lds32(c.sc + (row + 8) * c.PS + 4 * j));
    }
    fma_scaled<NT, RG>(acc, tmp, sl, sh);
  }
}

FP4X_DEV uint32_t w6_lane(uint32_t lo_src, uint32_t hi_src) {
  return (lo_src & 0x000F000Fu) | (hi_src & 0x00300030u) | 0x64006400u;
}

template <int NT, int RG>
FP4X_DEV void chunk_w6(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  const float zero[4] = {0.f, 0.f, 0.f, 0.f};
  const uint32_t kNeg1056 = 0xE420E420u;
  for (int j = 0; j < c.KC / 32; ++j) {
    uint32_t L[RG][2], Hs[RG][2];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int row = 16 * r + c.g + 8 * q;
        L[r][q] = lds32(c.a0 + row * c.P0 + 16 * j + 4 * c.tq);
        Hs[r][q] = prmt(lds16(c.a1 + row * c.P1 + 8 * j + 2 * c.tq), 0u, 0x4140u);
      }
    }
    float tmp[RG][NT][4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t b0[NT], b1[NT];
      load_b<NT>(c, 2 * j + h, b0, b1);
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        uint32_t A[4];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          uint32_t lo, hi;
          if (h == 0) {
            lo = w6_lane(L[r][q], Hs[r][q] << 4);          // elements r0, r4
            hi = w6_lane(L[r][q] >> 4, Hs[r][q]);          // r1, r5
          } else {
            lo = w6_lane(L[r][q] >> 8, Hs[r][q] << 2);     // r2, r6
            hi = w6_lane(L[r][q] >> 12, Hs[r][q] >> 2);    // r3, r7
          }
          A[q] = hadd2(lo, kNeg1056);
          A[2 + q] = hadd2(hi, kNeg1056);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          if (h == 0)
            mma_f16(tmp[r][t], A, b0[t], b1[t], zero);
          else
            mma_f16(tmp[r][t], A, b0[t], b1[t], tmp[r][t]);
        }
      }
    }
    float sl[RG], sh[RG];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int row = 16 * r + c.g;
      sl[r] = f16_bits_to_f32(lds16(c.sc + row * c.PS + 2 * j));
      sh[r] = f16_bits_to_f32(lds16(c.sc + (row + 8) * c.PS + 2 * j));
    }
    fma_scaled<NT, RG>(acc, tmp, sl, sh);
  }
}

template <int NT, int RG>
FP4X_DEV void chunk_nv4(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  for (int blk = 0; blk < c.KC / 128; ++blk) {
    uint4 a[RG][2];
    uint32_t sA[RG][2], sB[RG][2];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int row = 16 * r + c.g + 8 * q;
        a[r][q] = lds128(c.a0 + row * c.P0 + 64 * blk + 16 * c.tq);
        const uint32_t sf = e4m3x2_to_f16x2(lds16(c.sc + row * c.PS + 8 * blk + 2 * c.tq));
        sA[r][q] = prmt(sf, 0u, 0x1010u);
        sB[r][q] = prmt(sf, 0u, 0x3232u);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t b0[NT], b1[NT];
      load_b<NT>(c, 8 * blk + i, b0, b1);
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        uint32_t A[4];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const uint32_t wv = (i >> 1) == 0 ? a[r][q].x : (i >> 1) == 1 ? a[r][q].y : (i >> 1) == 2 ? a[r][q].z : a[r][q].w;
          const uint32_t hw = (i & 1) ? (wv >> 16) : wv;
          const uint32_t s2 = i < 4 ? sA[r][q] : sB[r][q];
          A[q] = hmul2(e2m1x2_to_f16x2(hw), s2);
          A[2 + q] = hmul2(e2m1x2_to_f16x2(hw >> 8), s2);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) mma_f16(acc[r][t], A, b0[t], b1[t], acc[r][t]);
      }
    }
  }
}

template <int NT, int RG>
FP4X_DEV void chunk_bf16(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  for (int u = 0; u < c.KC / 32; ++u) {
    uint4 a[RG][2];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      const int row = 16 * r + c.g;
      a[r][0] = lds128(c.a0 + row * c.P0 + 64 * u + 16 * c.tq);
      a[r][1] = lds128(c.a0 + (row + 8) * c.P0 + 64 * u + 16 * c.tq);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      uint32_t b0[NT], b1[NT];
      load_b<NT>(c, 2 * u + h, b0, b1);
#pragma unroll
      for (int r = 0; r < RG; ++r) {
        const uint32_t A[4] = {h ? a[r][0].z : a[r][0].x, h ? a[r][1].z : a[r][1].x, h ? a[r][0].w : a[r][0].y,
                               h ? a[r][1].w : a[r][1].y};
#pragma unroll
        for (int t = 0; t < NT; ++t) mma_bf16(acc[r][t], A, b0[t], b1[t], acc[r][t]);
      }
    }
  }
}

// INT2 group table: bytes T[c] (c = code) of bf16 values (-a, -b, +b, +a), a = bf16(1.5 s), b = bf16(0.5 s)
FP4X_DEV void int2_table(uint32_t s16, uint32_t& tlo, uint32_t& thi) {
  const float s = f16_bits_to_f32(s16);
  const uint32_t pk = pack_bf16x2(0.5f * s, 1.5f * s);  // bytes [b_lo, b_hi, a_lo, a_hi]
  tlo = prmt(pk, 0u, 0x2002u);
  thi = prmt(pk, 0u, 0x3113u) ^ 0x00008080u;
}

template <int NT, int RG>
FP4X_DEV void chunk_int2(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  const int gshift = c.group == 32 ? 1 : 0;
  for (int blk = 0; blk < c.KC / 256; ++blk) {
    uint4 a[RG][2];
#pragma unroll
    for (int r = 0; r < RG; ++r) {
      a[r][0] = lds128(c.a0 + (16 * r + c.g) * c.P0 + 64 * blk + 16 * c.tq);
      a[r][1] = lds128(c.a0 + (16 * r + c.g + 8) * c.P0 + 64 * blk + 16 * c.tq);
    }
#pragma unroll
    for (int gi = 0; gi < 4; ++gi) {
      // 16-k group index (within the chunk) of this thread's group gi, and its scale slot
      const int g16 = 16 * blk + 4 * c.tq + gi;
      const int sidx = g16 >> gshift;
      uint32_t tlo[RG][2], thi[RG][2], W[RG][2];
#pragma unroll
      for (int r = 0; r < RG; ++r) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int row = 16 * r + c.g + 8 * q;
          int2_table(lds16(c.sc + row * c.PS + 2 * sidx), tlo[r][q], thi[r][q]);
          W[r][q] = gi == 0 ? a[r][q].x : gi == 1 ? a[r][q].y : gi == 2 ? a[r][q].z : a[r][q].w;
        }
      }
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        uint32_t b0[NT], b1[NT];
        load_b<NT>(c, 16 * blk + 4 * gi + p, b0, b1);
#pragma unroll
        for (int r = 0; r < RG; ++r) {
          uint32_t A[4];
#pragma unroll
          for (int q = 0; q < 2; ++q) {
            const uint32_t z = (W[r][q] >> (2 * p)) & 0x03030303u;
            const uint32_t sl = z * 0x11u + 0x4040u;
            const uint32_t sh = __umulhi(z, 0x110000u) + 0x4040u;
            A[q] = prmt(tlo[r][q], thi[r][q], sl);
            A[2 + q] = prmt(tlo[r][q], thi[r][q], sh);
          }
#pragma unroll
          for (int t = 0; t < NT; ++t) mma_bf16(acc[r][t], A, b0[t], b1[t], acc[r][t]);
        }
      }
    }
  }
}

template <int FMT, int NT, int RG>
FP4X_DEV void compute_chunk(const ChunkCtx& c, float (&acc)[RG][NT][4]) {
  if (FMT == FMT_MX8) chunk_mx8<NT, RG>(c, acc);
  else if (FMT == FMT_W8) chunk_w8<NT, RG>(c, acc);
  else if (FMT == FMT_W6) chunk_w6<NT, RG>(c, acc);
  else if (FMT == FMT_NV4) chunk_nv4<NT, RG>(c, acc);
  else if (FMT == FMT_BF16) chunk_bf16<NT, RG>(c, acc);
  else chunk_int2<NT, RG>(c, acc);
}

// ------------------------------------------------------------------------------------------------------
// epilogues
// ------------------------------------------------------------------------------------------------------
// hyper-connection down epilogue (fused and unfused paths share it): di = bf16(v); bot = bf16(t*sigmoid(t)),
// t = bf16(f32(di) / hc), for columns < lr
FP4X_DEV void hc_down_store(__nv_bfloat16* di, __nv_bfloat16* bot, int N, int lr, int hc, int m, int n, float v) {
  const __nv_bfloat16 d = __float2bfloat16_rn(v);
  di[(int64_t)m * N + n] = d;
  if (n < lr && bot) {
    const float t = bf16_round(__bfloat162float(d) / (float)hc);
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

template <int EPI, int NT, int RG>
FP4X_DEV void run_epilogue(const GemvArgs& A, const GemvItem& it, int rt, const float (&v)[RG][NT][4], int g, int tq,
                           float* scr) {
  constexpr int RU = 16 * RG;
  if (EPI == EPI_STORE || EPI == EPI_HEAD || EPI == EPI_HC_DOWN) {
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int n = rt * RU + 16 * r + g + 8 * (e >> 1);
          const int m = 8 * t + 2 * tq + (e & 1);
          if (n < A.N && m < A.M) {
            if (EPI == EPI_HC_DOWN) {
              hc_down_store(reinterpret_cast<__nv_bfloat16*>(it.out), reinterpret_cast<__nv_bfloat16*>(it.out2),
                            A.N, A.lr, A.hc, m, n, v[r][t][e]);
            } else {
              const float val = v[r][t][e] * A.post;
              store_out(it.out, A.out_dtype, (int64_t)m * A.out_stride + n, val);
              if (EPI == EPI_HEAD && it.out2)
                reinterpret_cast<__nv_bfloat16*>(it.out2)[(int64_t)m * A.out_stride + n] = __float2bfloat16_rn(val);
            }
          }
        }
  } else {  // EPI_HC_UP: rows of this unit are hc streams x bj columns (interleaved); RU == hc * bj
    constexpr int MPx = 8 * NT;
    const int lane = g * 4 + tq;
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int row = 16 * r + g + 8 * (e >> 1);
          const int m = 8 * t + 2 * tq + (e & 1);
          const float gl = bf16_round(v[r][t][e]);
          scr[row * MPx + m] = bf16_round(sigmoidf_(gl));
        }
    __syncwarp();
    const int bj = A.bj, hc = A.hc;
    const int H = A.N / hc;
    const __nv_bfloat16* nrm = reinterpret_cast<const __nv_bfloat16*>(A.nrm);
    for (int o = lane; o < bj * A.M; o += 32) {
      const int m = o / bj, c = o - m * bj;
      const int col = rt * bj + c;
      float nv[8], gv[8];
      for (int s = 0; s < hc; ++s) {
        nv[s] = __bfloat162float(nrm[(int64_t)m * A.nrm_stride + s * H + col]);
        gv[s] = scr[(s * bj + c) * MPx + m];
      }
      reinterpret_cast<__nv_bfloat16*>(it.out)[(int64_t)m * A.out_stride + col] =
          __float2bfloat16_rn(hc_gate_mean(nv, gv, hc));
    }
    __syncwarp();
  }
}

// ------------------------------------------------------------------------------------------------------
// the kernel
// ------------------------------------------------------------------------------------------------------
template <int FMT>
FP4X_DEV void issue_chunk(const GemvArgs& A, const GemvItem& it, int64_t u, int k_panel0, uint32_t stage,
                          uint32_t bar, int lane, int RU) {
  constexpr FmtGeom G = fmt_geom(FMT);
  const int rt = (int)(u / A.NCH), c = (int)(u - (int64_t)rt * A.NCH);
  const int k0 = k_panel0 + c * A.KC;
  const int pb0 = A.KC * G.n0 / G.d0;
  const int pb1 = G.n1 ? A.KC * G.n1 / G.d1 : 0;
  const int sd = FMT == FMT_INT2 ? A.group / 2 : G.sd;
  const int sbytes = G.sn ? A.KC * G.sn / sd : 0;
  if (lane == 0) mbar_arrive_expect_tx(bar, (uint32_t)(RU * (pb0 + pb1)));
  __syncwarp();
  const int row0 = rt * RU;
  for (int r = lane; r < RU; r += 32) {
    const int row = min(row0 + r, A.N - 1);
    bulk_g2s(stage + r * A.P0, it.p0 + (int64_t)row * A.ld0 + (int64_t)k0 * G.n0 / G.d0, pb0, bar);
    if constexpr (G.n1 != 0) bulk_g2s(stage + RU * A.P0 + r * A.P1, it.p1 + (int64_t)row * A.ld1 + (int64_t)k0 * G.n1 / G.d1, pb1, bar);
  }
  if constexpr (G.sn != 0) {
    const int wpr = sbytes / 4;
    const uint32_t sbase = stage + RU * (A.P0 + A.P1);
    const int64_t koff = (int64_t)k0 * G.sn / sd;
    for (int w = lane; w < RU * wpr; w += 32) {
      const int r = w / wpr, cw = w - r * wpr;
      const int row = min(row0 + r, A.N - 1);
      cp_async4(sbase + r * A.PS + 4 * cw, it.sc + (int64_t)row * A.lds + koff + 4 * cw);
    }
  }
  cp_async_arrive_noinc(bar);
}

template <int FMT, int NT, int RG, int EPI>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const __grid_constant__ GemvArgs A) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int RU = 16 * RG;
  constexpr int MP = 8 * NT;
  constexpr FmtGeom G = fmt_geom(FMT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, tq = lane & 3;
  const int p = blockIdx.y, b = blockIdx.z;
  GemvItem it = A.item;
  if (A.items4) {
    const void* const* e = A.items4 + 4 * b;
    it.x = e[0];
    it.p0 = (const uint8_t*)e[1];
    it.sc = (const uint8_t*)e[2];
    it.out = (void*)e[3];
  }
  const int k_panel0 = p * A.KPW;

  const uint32_t bars = smem_u32(smem) + warp * kMaxStages * 8;
  const uint32_t stages = smem_u32(smem + A.smem_stage) + warp * A.NS * A.STG;
  const int Wp = A.CPP * kWarps;
  const int wg = blockIdx.x * kWarps + warp;
  const int64_t Up = (int64_t)A.RT * A.NCH;
  const int64_t u_begin = A.whole ? range_begin(A.RT, Wp, wg) * A.NCH : range_begin(Up, Wp, wg);
  const int64_t u_end = A.whole ? range_begin(A.RT, Wp, wg + 1) * A.NCH : range_begin(Up, Wp, wg + 1);

  if (lane == 0) {
    for (int s = 0; s < A.NS; ++s) mbar_init(bars + 8 * s, 33);
    mbar_init_fence();
  }
  __syncwarp();
  for (int64_t q = 0; q < A.NS && u_begin + q < u_end; ++q)
    issue_chunk<FMT>(A, it, u_begin + q, k_panel0, stages + (uint32_t)q * A.STG, bars + 8 * (uint32_t)q, lane, RU);

  pdl_wait();
  stage_activations<FMT>(A, it, smem, MP, k_panel0);
  __syncthreads();
  pdl_launch_dependents();

  const float* xsc = reinterpret_cast<const float*>(smem + kWarps * kMaxStages * 8);
  float* scr = reinterpret_cast<float*>(smem + A.smem_scr) + warp * RU * MP;
  ChunkCtx cc;
  cc.P0 = A.P0; cc.P1 = A.P1; cc.PS = A.PS; cc.KC = A.KC; cc.XP = A.XP; cc.g = g; cc.tq = tq; cc.group = A.group;
  const uint32_t xrow = smem_u32(smem + A.smem_x) + g * A.XP + tq * 8;

  float acc[RG][NT][4];
  zero_acc<NT, RG>(acc);
  int cur_rt = -1;
  bool ok = true;

  auto flush = [&](int rt) {
    // remove the activation scale (exact power of two) per token column
    if (G.xf16) {
#pragma unroll
      for (int r = 0; r < RG; ++r)
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[r][t][e] *= xsc[MP + 8 * t + 2 * tq + (e & 1)];
    }
    const int64_t uf = (int64_t)rt * A.NCH, ul = uf + A.NCH - 1;
    const int wf = A.whole ? wg : owner_of(uf, Up, Wp), wl = A.whole ? wg : owner_of(ul, Up, Wp);
    const int segs = wl - wf + 1;
    if (A.KP == 1 && segs == 1) {
      run_epilogue<EPI, NT, RG>(A, it, rt, acc, g, tq, scr);
      return;
    }
    auto slot_of = [&](int pp, int w) -> int64_t {
      if (A.KP == 1) {  // at most two shared tiles per warp: its first (slot 0) and last (slot 1)
        const int first_rt = (int)(range_begin(Up, Wp, w) / A.NCH);
        return ((int64_t)b * Wp + w) * 2 + (rt == first_rt ? 0 : 1);
      }
      return (((int64_t)b * A.KP + pp) * A.RT + rt) * A.SMAX + (w - wf);
    };
    float* mine = A.ws + slot_of(p, wg) * (RU * MP);
#pragma unroll
    for (int r = 0; r < RG; ++r)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int row = 16 * r + g, m = 8 * t + 2 * tq;
        __stcg(reinterpret_cast<float2*>(mine + row * MP + m), make_float2(acc[r][t][0], acc[r][t][1]));
        __stcg(reinterpret_cast<float2*>(mine + (row + 8) * MP + m), make_float2(acc[r][t][2], acc[r][t][3]));
      }
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) {
      const int old = atomicAdd(A.sem + (int64_t)b * A.RT + rt, 1);
      last = (old == A.KP * segs - 1);
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    if (!last) return;
    __threadfence();
    float tot[RG][NT][4];
    zero_acc<NT, RG>(tot);
    for (int pp = 0; pp < A.KP; ++pp)
      for (int w = wf; w <= wl; ++w) {
        const float* src = A.ws + slot_of(pp, w) * (RU * MP);
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const int row = 16 * r + g, m = 8 * t + 2 * tq;
            const float2 lo = __ldcg(reinterpret_cast<const float2*>(src + row * MP + m));
            const float2 hi = __ldcg(reinterpret_cast<const float2*>(src + (row + 8) * MP + m));
            tot[r][t][0] += lo.x; tot[r][t][1] += lo.y; tot[r][t][2] += hi.x; tot[r][t][3] += hi.y;
          }
      }
    run_epilogue<EPI, NT, RG>(A, it, rt, tot, g, tq, scr);
    if (lane == 0) atomicExch(A.sem + (int64_t)b * A.RT + rt, 0);
  };

  for (int64_t u = u_begin; u < u_end; ++u) {
    const int64_t q = u - u_begin;
    const int st = (int)(q % A.NS);
    const uint32_t parity = (uint32_t)((q / A.NS) & 1);
    const int rt = (int)(u / A.NCH), c = (int)(u - (int64_t)rt * A.NCH);
    if (rt != cur_rt) {
      if (cur_rt >= 0) flush(cur_rt);
      zero_acc<NT, RG>(acc);
      cur_rt = rt;
    }
    if (!mbar_wait_bounded(bars + 8 * st, parity, A.err)) { ok = false; break; }
    const uint32_t sbase = stages + (uint32_t)st * A.STG;
    cc.a0 = sbase;
    cc.a1 = sbase + RU * A.P0;
    cc.sc = sbase + RU * (A.P0 + A.P1);
    cc.xb = xrow + c * (A.KC / 16) * 32;
    compute_chunk<FMT, NT, RG>(cc, acc);
    fence_proxy_async_smem();
    __syncwarp();
    if (u + A.NS < u_end) issue_chunk<FMT>(A, it, u + A.NS, k_panel0, sbase, bars + 8 * st, lane, RU);
  }
  if (ok && cur_rt >= 0) flush(cur_rt);
  if (!ok) {
    // a stage never completed (error already recorded): wait, bounded, for the copies this warp still has in
    // flight so that nothing lands in shared memory after the CTA has gone, then leave
    asm volatile("cp.async.wait_all;" ::: "memory");
    for (int s = 0; s < A.NS; ++s) {
      uint32_t par = 0;
      while (par < 2 && !mbar_try_wait(bars + 8 * s, par)) ++par;
    }
    const uint64_t t0 = global_ns();
    while (global_ns() - t0 < 100000000ull) {
      bool all = true;
      for (int s = 0; s < A.NS; ++s) all = all && (mbar_try_wait(bars + 8 * s, 0) || mbar_try_wait(bars + 8 * s, 1));
      if (all) break;
    }
  }
}

}  // namespace fp4x
