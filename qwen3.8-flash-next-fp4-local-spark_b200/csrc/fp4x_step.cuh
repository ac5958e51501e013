// Persistent decode-step kernel: one launch runs an ordered list of GEMV-family ops (a decode step's quantized
// linears and hyper-connection mixers) with one CTA per SM.
//
//   * Every CTA walks the op list in order and takes the same stream-K share of each op that a standalone launch
//     with one CTA per SM would (row blocks x k chunks, split evenly; split row blocks are summed by their last
//     arriving warp in a fixed order, so results do not depend on timing).
//   * The producer warp streams the weight tiles of all the CTA's ops, one op after the other, through a single
//     ring of shared-memory stages.  Weights never depend on earlier ops, so it never waits for data: while the
//     consumer warps finish op j (or wait for its inputs), the stages of op j+1, j+2, ... are already landing.
//   * The consumer warps of an op first wait until every op it depends on is complete (a per-op counter of CTAs
//     that finished it, read with acquire semantics), then stage their k range of the activations from L2, consume
//     the stages and run the op's epilogue.  Dependencies are the read/write hazards between the ops' activation
//     and output buffers, found on the host when the step is prepared.
//   * Every wait is bounded (2 s) and gives up when another CTA has already recorded an error, so a fault in one
//     op ends the whole launch quickly; the counters are then left for the host to zero (fp4x_device_error).
#pragma once
#include "fp4x_gemv.cuh"

namespace fp4x {

constexpr int kStepMaxDeps = 6;
constexpr int kStepMaxStages = 12;
constexpr int kStepSlotBytes = 18432;  // stage pitch: the largest stage of the step formats (NVFP4, 64 x 288 bytes)

// One op of a step: the standalone GEMV's argument block (geometry, TMA descriptors, pointers, plan) plus the
// dispatch keys and dependencies.  In a step, a.STG is the ring's stage pitch and a.CPP the number of CTAs that
// share the op's units.
struct alignas(64) StepOp {
  GemvArgs a;
  int fmt, epi, shape;
  int ndeps;
  int deps[kStepMaxDeps];
};

struct StepArgs {
  const StepOp* ops;
  int nops;
  int NS;              // ring stages
  int SLOT;            // stage pitch (bytes, multiple of 1024): kStepSlotBytes
  int smem_x, smem_xraw, smem_misc, smem_scr, smem_comb;
  int* done;           // [nops] CTAs that finished each op; zero on entry, zeroed again by the last CTA to finish
  int* fin;            // CTAs that finished the whole step
  int* err;            // device error word
  uint64_t* trace;     // optional timeline: [grid][nops][8] globaltimer stamps written by consumer thread 0: op
                       // start, inputs ready, staged, done, first weight stage ready, stage loop done, last flush
                       // done; null when off
};

FP4X_DEV void step_stamp(const StepArgs& S, int j, int what) {
  if (S.trace && threadIdx.x == 0) S.trace[((int64_t)blockIdx.x * S.nops + j) * 8 + what] = global_ns();
}

FP4X_DEV int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
FP4X_DEV int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

// mbarrier wait that gives up after 2 s, or at once when the error word is set (another CTA gave up)
FP4X_DEV bool step_wait(uint32_t bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0) {
      if (ld_volatile(err)) return false;
      if (global_ns() - t0 > 2000000000ull) {
        set_dev_error(err, kDevWaitTimeout);
        return false;
      }
    }
  }
}

// the unit range [u_begin, u_end) of CTA `cta` in an op: the op's units are split over its first A.CPP CTAs
// (min(CTAs, units): every one of them owns at least one unit); whole plans take whole row blocks
FP4X_DEV void step_units(const GemvArgs& A, int cta, int64_t& ub, int64_t& ue) {
  const int W = A.CPP;
  if (cta >= W) {
    ub = ue = 0;
  } else if (A.whole) {
    ub = range_begin(A.RT, W, cta) * A.NCH;
    ue = range_begin(A.RT, W, cta + 1) * A.NCH;
  } else {
    const int64_t Up = (int64_t)A.RT * A.NCH;
    ub = range_begin(Up, W, cta);
    ue = range_begin(Up, W, cta + 1);
  }
}

// ---------------------------------------------------------------------------------------------------------------
// producer: the weight tiles of one op's units into the ring (the standalone producer loop, ring state carried over)
// ---------------------------------------------------------------------------------------------------------------
template <int FMT>
__device__ __noinline__ bool step_produce(const GemvArgs& A, int64_t ub, int64_t ue, uint8_t* base, int SLOT, int NS, uint32_t full0,
                           uint32_t empty0, int& s, int& round, int& issued, int* err) {
  constexpr FmtGeom G = fmt_geom(FMT);
  const int lane = threadIdx.x & 31;
  const int tx = kRB * (A.NB0 * A.BI0 + (G.n1 ? A.BI1 : 0));
  const int scw = A.scw;
  const int words_per_row = G.sn ? A.SB / scw : 0;
  const int sd = G.sd;
  int blk = (int)(ub / A.NCH), chunk = (int)(ub - (int64_t)blk * A.NCH);
  for (int64_t q = ub; q < ue; ++q) {
    if (round > 0 && !step_wait(empty0 + 8 * s, (uint32_t)((round - 1) & 1), err)) return false;
    const int k0 = chunk * A.KC;
    const uint32_t stage = smem_u32(base) + (uint32_t)s * SLOT;
    const uint32_t bar = full0 + 8 * s;
    if (lane == 0) {
      mbar_arrive_expect_tx(bar, (uint32_t)tx);
      const int xb0 = k0 * G.n0 / G.d0;
      for (int bx = 0; bx < A.NB0; ++bx) tma_load_2d(stage + bx * kRB * A.BI0, &A.tm0, xb0 + bx * A.BI0, blk * kRB, bar);
      if constexpr (G.n1 != 0) tma_load_2d(stage + A.off_p1, &A.tm1, k0 * G.n1 / G.d1, blk * kRB, bar);
    }
    if constexpr (G.sn != 0) {
      const int64_t koff = (int64_t)k0 * G.sn / sd;
      const uint32_t sbase = stage + A.off_sc;
      for (int w = lane; w < kRB * words_per_row; w += 32) {
        const int r = w / words_per_row, cw = w - r * words_per_row;
        const int row = min(blk * kRB + r, A.N - 1);
        const uint8_t* src = A.item.sc + (int64_t)row * A.lds + koff + (int64_t)cw * scw;
        const uint32_t dst = sbase + r * A.SB + cw * scw;
        if (scw == 16) cp_async16(dst, src);
        else if (scw == 8) cp_async8(dst, src);
        else cp_async4(dst, src);
      }
    }
    cp_async_arrive_noinc(bar);
    ++issued;
    if (++s == NS) { s = 0; ++round; }
    if (++chunk == A.NCH) { chunk = 0; ++blk; }
  }
  return true;
}

// ---------------------------------------------------------------------------------------------------------------
// activation staging of a k range: chunks c_lo .. c_lo + nc - 1 (mod NCH) of the op's K.  Every consumer thread
// issues its 16-byte asynchronous copies of the raw bf16 rows at once (L2 only: other SMs wrote them), so the
// staging costs one L2 round trip; then the rows are converted from shared memory into a local panel of nc chunks
// in the format's permuted B order.
// ---------------------------------------------------------------------------------------------------------------
template <int FMT>
FP4X_DEV void step_stage(const GemvArgs& A, uint8_t* base, int smem_x, int smem_xraw, int smem_misc, int XP, int c_lo,
                         int nc) {
  constexpr FmtGeom G = fmt_geom(FMT);
  constexpr int nthr = kCWarps * 32;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(A.item.x);
  const int64_t xs = A.x_stride;
  const int kloc = nc * A.KC;   // local k extent
  const int vpr = kloc / 8;     // 16-byte vectors per token row
  const uint32_t raw = smem_u32(base + smem_xraw);
  for (int i = tid; i < A.M * vpr; i += nthr) {
    const int tok = i / vpr, lk = (i - tok * vpr) * 8;
    const int lc = lk / A.KC;
    int c = c_lo + lc;
    if (c >= A.NCH) c -= A.NCH;
    cp_async16(raw + (uint32_t)(tok * kloc + lk) * 2u, x + (int64_t)tok * xs + c * A.KC + (lk - lc * A.KC));
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  named_bar(1, nthr);
  const __nv_bfloat16* xr = reinterpret_cast<const __nv_bfloat16*>(base + smem_xraw);
  float* xsc = reinterpret_cast<float*>(base + smem_misc);  // [8] scale, [8] inverse (per token)
  if (G.xf16) {
    for (int tok = warp; tok < A.M; tok += kCWarps) {
      float mx = 0.f;
      const uint4* row = reinterpret_cast<const uint4*>(xr + (int64_t)tok * kloc);
      for (int i = lane; i < vpr; i += 32) {
        const uint4 v = row[i];
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          mx = fmaxf(mx, fabsf(bf16_bits_to_f32(w[e] & 0xffffu)));
          mx = fmaxf(mx, fabsf(bf16_bits_to_f32(w[e] >> 16)));
        }
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) {
        int t = 0;
        const uint32_t bits = __float_as_uint(mx);
        if (mx > 0.f && (bits >> 23) < 255u) {
          t = 14 - ((int)(bits >> 23) - 127);
          t = t < -113 ? -113 : (t > 126 ? 126 : t);
        }
        xsc[tok] = __uint_as_float((uint32_t)(127 + t) << 23);
        xsc[8 + tok] = __uint_as_float((uint32_t)(127 - t) << 23);
      }
    }
    named_bar(1, nthr);
  }
  const uint32_t xbase = smem_u32(base + smem_x);
  const int nblk = kloc / G.qb;
  for (int i = tid; i < A.M * nblk; i += nthr) {
    const int tok = i / nblk, lb = i - tok * nblk;
    const float scl = G.xf16 ? xsc[tok] : 1.f;
    uint32_t v[4] = {0, 0, 0, 0};
    const uint32_t src = raw + (uint32_t)(tok * kloc + lb * G.qb) * 2u;
    if (G.qb == 4) {
      const uint2 t = lds64(src);
      v[0] = t.x; v[1] = t.y;
    } else {
      const uint4 t = lds128(src);
      v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
    }
    int sp[4];
    int tq;
    stage_block_positions<FMT>(lb, sp, tq);
    const uint32_t trow = xbase + tok * XP;
    if (G.qb == 4) {
      sts64(trow + sp[0] * 32 + tq * 8, cvt_pair(v[0], scl, G.xf16), cvt_pair(v[1], scl, G.xf16));
    } else {  // W6: elements r0..r7; quads (r0,r4,r1,r5) and (r2,r6,r3,r7)
      sts64(trow + sp[0] * 32 + tq * 8, cvt_pair(pick2(v[0], 0, v[2], 0), scl, G.xf16),
            cvt_pair(pick2(v[0], 1, v[2], 1), scl, G.xf16));
      sts64(trow + sp[1] * 32 + tq * 8, cvt_pair(pick2(v[1], 0, v[3], 0), scl, G.xf16),
            cvt_pair(pick2(v[1], 1, v[3], 1), scl, G.xf16));
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// epilogues: the standalone ones, except that the hyper-connection up epilogue synchronises its warp pair (32
// interleaved rows = 8 output columns x 4 streams) through an mbarrier with a bounded wait instead of a named
// barrier, so a warp that stopped on an error cannot leave its partner waiting for ever
// ---------------------------------------------------------------------------------------------------------------
FP4X_DEV bool pair_sync(uint32_t bar, uint32_t& count, int* err) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
  const bool ok = step_wait(bar, count & 1u, err);
  ++count;
  __syncwarp();
  return ok;
}

template <int EPI, int NT>
FP4X_DEV bool step_epilogue(const GemvArgs& A, int row0, const float (&v)[NT][4], int warp, int g, int tq,
                            float* scr_all, uint32_t pair0, uint32_t& npair, int* err) {
  if (EPI != EPI_HC_UP) {
    run_epilogue<EPI, NT>(A, A.item, row0, v, warp, g, tq, scr_all);
    return true;
  }
  constexpr int MP = 8 * NT;
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
  const uint32_t bar = pair0 + 8 * (warp >> 1);
  if (rows == 32) {
    first_warp = warp & ~1;
    nwarps = 2;
    if (!pair_sync(bar, npair, err)) return false;
  } else {
    __syncwarp();
  }
  const float* bscr = scr_all + first_warp * 16 * MP;
  const int blk_row0 = row0 - 16 * (warp - first_warp);
  if (blk_row0 < A.N) {
    const int jb = blk_row0 / rows;
    const int H = A.N / A.hc;
    const __nv_bfloat16* nrm = reinterpret_cast<const __nv_bfloat16*>(A.nrm);
    const int nout = A.bj * A.M;
    for (int o = lane + 32 * (warp - first_warp); o < nout; o += 32 * nwarps) {
      const int m = o / A.bj, cidx = o - m * A.bj;
      const int col = jb * A.bj + cidx;
      float nv[8], gv[8];
      for (int s = 0; s < A.hc; ++s) {
        nv[s] = __bfloat162float(nrm[(int64_t)m * A.nrm_stride + s * H + col]);
        gv[s] = bscr[(s * A.bj + cidx) * MP + m];
      }
      reinterpret_cast<__nv_bfloat16*>(A.item.out)[(int64_t)m * A.out_stride + col] =
          __float2bfloat16_rn(hc_gate_mean(nv, gv, A.hc));
    }
  }
  if (rows == 32) return pair_sync(bar, npair, err);
  __syncwarp();
  return true;
}

// ---------------------------------------------------------------------------------------------------------------
// consumer: one op's units of this CTA (wait for dependencies, stage, compute, reduce, epilogue)
// ---------------------------------------------------------------------------------------------------------------
struct StepConsumerState {
  int s;
  uint32_t phase;
  uint32_t nflush;
  uint32_t npair;  // hyper-connection up: warp-pair handshakes so far (mbarrier parity)
  int consumed;    // stages this warp has taken from the ring
};

// stage geometry of each format in a step (compile-time, so the hot loop keeps no geometry in registers)
template <int FMT>
struct StepGeom {
  static constexpr int KC = FMT == FMT_NV4 ? 512 : 256;            // k per stage
  static constexpr int NB0 = FMT == FMT_W6 ? 1 : 2;                // 128-byte plane-0 boxes per stage
  static constexpr int BI1 = FMT == FMT_W6 ? 64 : 0;               // plane-1 box bytes
  static constexpr int SB = FMT == FMT_NV4 ? 32 : (FMT == FMT_MX8 ? 8 : 16);  // scale bytes per row
  static constexpr int SHAPE = FMT == FMT_W6 ? SHAPE_128x1 : SHAPE_128x2;
  static constexpr int OFF_P1 = kRB * NB0 * 128;
  static constexpr int OFF_SC = OFF_P1 + kRB * BI1;
};

// Split-K flush of one row block (k-group hand-over, partial slot, last-arriver sum, epilogue); out of line so
// that the stage loop keeps none of its state in registers.
template <int FMT, int EPI>
__device__ __noinline__ bool step_flush(const StepArgs& S, const StepOp& op, int blk, float (&acc)[1][4],
                                        uint8_t* base, uint32_t comb_full0, uint32_t comb_empty0,
                                        StepConsumerState& st) {
  constexpr FmtGeom G = fmt_geom(FMT);
  constexpr int NT = 1, MP = 8;
  const GemvArgs& A = op.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int wrow = warp & (kRW - 1), kg = warp / kRW;
  const int cta = blockIdx.x, CPP = A.CPP;
  float* comb = reinterpret_cast<float*>(base + S.smem_comb) + (wrow * 32 + lane) * (NT * 4);
  const uint32_t pair0 = comb_empty0 + 8 * kRW;  // two warp-pair barriers after the k-group handshakes
  float* scr = reinterpret_cast<float*>(base + S.smem_scr);
  const uint32_t cf_bar = comb_full0 + 8 * wrow, ce_bar = comb_empty0 + 8 * wrow;
  const uint32_t par = st.nflush & 1u;
  ++st.nflush;
  if (kg == 1) {
    if (st.nflush > 1 && !step_wait(ce_bar, par ^ 1u, S.err)) return false;
    *reinterpret_cast<float4*>(comb) = make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]);
    __syncwarp();
    if (lane == 0) mbar_arrive(cf_bar);
    return true;
  }
  if (!step_wait(cf_bar, par, S.err)) return false;
  {
    const float4 o = *reinterpret_cast<const float4*>(comb);
    acc[0][0] += o.x; acc[0][1] += o.y; acc[0][2] += o.z; acc[0][3] += o.w;
  }
  __syncwarp();
  if (lane == 0) mbar_arrive(ce_bar);
  if (G.xf16) {
    const float* xsc = reinterpret_cast<const float*>(base + S.smem_misc);
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[0][e] *= xsc[8 + 2 * tq + (e & 1)];
  }
  const int row0 = blk * kRB + 16 * wrow;
  const int Up = A.whole ? A.RT : A.RT * A.NCH;
  int cf, cl;
  if (A.whole) {
    cf = cl = cta;
  } else {
    const int uf = blk * A.NCH, ul = uf + A.NCH - 1;
    cf = owner_of(uf, Up, CPP);
    cl = owner_of(ul, Up, CPP);
  }
  const int segs = cl - cf + 1;
  if (segs == 1) return step_epilogue<EPI, NT>(A, row0, acc, wrow, g, tq, scr, pair0, st.npair, S.err);
  auto slot_of = [&](int cc) -> int64_t {  // a CTA shares at most two blocks: its first (slot 0) and last (1)
    const int first_blk = (int)(range_begin(Up, CPP, cc) / A.NCH);
    return ((int64_t)cc * 2 + (blk == first_blk ? 0 : 1)) * kRW + wrow;
  };
  float* mine = A.ws + slot_of(cta) * (16 * MP);
  __stcg(reinterpret_cast<float2*>(mine + g * MP + 2 * tq), make_float2(acc[0][0], acc[0][1]));
  __stcg(reinterpret_cast<float2*>(mine + (g + 8) * MP + 2 * tq), make_float2(acc[0][2], acc[0][3]));
  __syncwarp();
  int* semp = A.sem + blk * kRW + wrow;
  int last = 0;
  if (lane == 0) last = (atomic_add_acq_rel(semp, 1) == segs - 1);
  last = __shfl_sync(0xffffffffu, last, 0);
  __syncwarp();
  if (!last) return true;
  float tot[1][4] = {{0.f, 0.f, 0.f, 0.f}};
  constexpr int kBatch = 16;  // every slot load of a batch is in flight before the first is added
  for (int i0 = 0; i0 < segs; i0 += kBatch) {
    float2 v[kBatch][2];
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (i0 + j < segs) {
        const float* src = A.ws + slot_of(cf + i0 + j) * (16 * MP);
        v[j][0] = __ldcg(reinterpret_cast<const float2*>(src + g * MP + 2 * tq));
        v[j][1] = __ldcg(reinterpret_cast<const float2*>(src + (g + 8) * MP + 2 * tq));
      }
    }
#pragma unroll
    for (int j = 0; j < kBatch; ++j) {
      if (i0 + j < segs) {
        tot[0][0] += v[j][0].x; tot[0][1] += v[j][0].y;
        tot[0][2] += v[j][1].x; tot[0][3] += v[j][1].y;
      }
    }
  }
  const bool ok = step_epilogue<EPI, NT>(A, row0, tot, wrow, g, tq, scr, pair0, st.npair, S.err);
  if (lane == 0) atomicExch(semp, 0);
  return ok;
}

// One op's units of this CTA: wait for the op's dependencies, stage the activations, consume the weight stages and
// flush each row block.  The ring position and the flush / pair counters carry over from op to op in `st`.
template <int FMT, int EPI>
__device__ __noinline__ bool step_consume(const StepArgs& S, const StepOp& op, int ub, int ue, uint8_t* base,
                                          uint32_t full0, uint32_t empty0, uint32_t comb_full0,
                                          uint32_t comb_empty0, StepConsumerState& st) {
  using SG = StepGeom<FMT>;
  constexpr int NT = 1;
  const GemvArgs& A = op.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int wrow = warp & (kRW - 1), kg = warp / kRW;
  const int grid = gridDim.x;
  const int nunits = ue - ub;
  const int NCH = A.NCH;
  int* abort_flag = reinterpret_cast<int*>(base + S.smem_misc + 64);

  // 1. dependencies: thread 0 waits until every op this one depends on has been finished by all CTAs
  if (threadIdx.x == 0) {
    int bad = 0;
    for (int d = 0; d < op.ndeps && !bad; ++d) {
      const int* cnt = S.done + op.deps[d];  // every CTA of the grid counts itself in when it is done with an op
      if (ld_acquire_gpu(cnt) >= grid) continue;
      const uint64_t t0 = global_ns();
      for (uint32_t it = 1;; ++it) {
        if (ld_acquire_gpu(cnt) >= grid) break;
        if ((it & 63u) == 0) {
          if (ld_volatile(S.err)) { bad = 1; break; }
          if (global_ns() - t0 > 2000000000ull) {
            set_dev_error(S.err, kDevWaitTimeout);
            bad = 1;
            break;
          }
        }
      }
    }
    *abort_flag = bad;
  }
  named_bar(1, kCWarps * 32);
  if (*reinterpret_cast<volatile int*>(abort_flag)) return false;
  step_stamp(S, (int)(&op - S.ops), 1);

  // 2. activations of the CTA's k range
  int c_lo = 0, nc = NCH;
  if (!A.whole && nunits < NCH) {
    c_lo = ub % NCH;
    nc = nunits;
  }
  constexpr int kSteps = SG::KC / 16;  // mma k-steps per stage
  const int XP = nc * kSteps * 32 + 32;
  step_stage<FMT>(A, base, S.smem_x, S.smem_xraw, S.smem_misc, XP, c_lo, nc);
  named_bar(1, kCWarps * 32);
  step_stamp(S, (int)(&op - S.ops), 2);

  // 3. the stage loop: geometry is compile-time; the loop keeps the ring position, the chunk and the warp context
  WarpCtx wc;
  wc.BI0 = 128; wc.BI1 = SG::BI1; wc.NB0 = SG::NB0; wc.SB = SG::SB; wc.XP = XP; wc.CPB = 8;
  wc.g = g; wc.tq = tq; wc.rbase = 16 * wrow;
  wc.gshift = 0;
  {
    const int r = 16 * wrow + (lane & 7) + 8 * ((lane >> 3) & 1);
    wc.lrow0 = (uint32_t)(r * 128);
    wc.lswz = r & 7;
    wc.lsel = lane >> 4;
  }
  // B rows at or beyond M read token M-1 (only M rows are staged; those columns are never stored)
  const int grow = g < A.M ? g : A.M - 1;
  const uint32_t xrow = smem_u32(base + S.smem_x) + grow * XP + tq * 8;
  const uint32_t ring = smem_u32(base);
  const int NS = S.NS;
  int* err = S.err;
  int s = st.s;
  uint32_t phase = st.phase;
  float acc[NT][4];
  zero4<NT>(acc);
  int blk = ub / NCH, chunk = ub - blk * NCH;
  int cur = blk;
  bool ok = true;
  for (int q = ub; q < ue; ++q) {
    if (blk != cur) {
      st.s = s;
      st.phase = phase;
      ok = step_flush<FMT, EPI>(S, op, cur, acc, base, comb_full0, comb_empty0, st);
      if (!ok) break;
      zero4<NT>(acc);
      cur = blk;
    }
    if (!step_wait(full0 + 8 * s, phase, err)) { ok = false; break; }
    if (q == ub) step_stamp(S, (int)(&op - S.ops), 4);
    const uint32_t stage = ring + (uint32_t)s * kStepSlotBytes;
    wc.p0 = stage;
    wc.p1 = stage + SG::OFF_P1;
    wc.sc = stage + SG::OFF_SC;
    int lc = chunk - c_lo;
    if (lc < 0) lc += NCH;
    wc.xb = xrow + lc * kSteps * 32;
    compute_stage<FMT, NT, SG::SHAPE>(wc, kg, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * s);
    ++st.consumed;
    if (++s == NS) { s = 0; phase ^= 1u; }
    if (++chunk == NCH) { chunk = 0; ++blk; }
  }
  st.s = s;
  st.phase = phase;
  step_stamp(S, (int)(&op - S.ops), 5);
  if (ok) ok = step_flush<FMT, EPI>(S, op, cur, acc, base, comb_full0, comb_empty0, st);
  step_stamp(S, (int)(&op - S.ops), 6);
  return ok;
}

// the (format, epilogue, shape) combinations a step runs
enum StepKind : int {
  STEP_NV4 = 0,      // NVFP4, store (post-scale gs), two 128-byte boxes per stage
  STEP_W6 = 1,       // W6 g32, store, one 128-byte box
  STEP_W8 = 2,       // W8 g64, store, two boxes
  STEP_HC_DOWN = 3,  // W8 g64, hyper-connection down epilogue, two boxes
  STEP_HC_UP = 4,    // W8 g64, hyper-connection up epilogue (whole row blocks), two boxes
  STEP_MX8 = 5,      // MXFP8, store, two boxes
  STEP_KINDS = 6
};

// 288 threads in one CTA per SM: the 9 warps spread over the 4 SM sub-partitions put 3 warps on one of them, whose
// 16K-register share then bounds a thread at 168 registers (__launch_bounds__ derives that).
template <int NT>
__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepArgs S) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  uint8_t* base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5;
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + S.smem_misc + 128);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStepMaxStages);
  const uint32_t comb_full0 = smem_u32(bars + 2 * kStepMaxStages), comb_empty0 = comb_full0 + 8 * kRW;
  if (threadIdx.x == 0) {
    for (int s = 0; s < S.NS; ++s) {
      mbar_init(full0 + 8 * s, 33);
      mbar_init(empty0 + 8 * s, kCWarps);
    }
    for (int i = 0; i < kRW; ++i) {
      mbar_init(comb_full0 + 8 * i, 1);
      mbar_init(comb_empty0 + 8 * i, 1);
    }
    for (int i = 0; i < kRW / 2; ++i) mbar_init(comb_empty0 + 8 * (kRW + i), 2);
    *reinterpret_cast<volatile int*>(base + S.smem_misc + 68) = 0;
    mbar_init_fence();
  }
  __syncthreads();
  const int cta = blockIdx.x, G = gridDim.x;
  int* issued = reinterpret_cast<int*>(base + S.smem_misc + 68);  // stages the producer issued (drain on abort)

  if (warp == kCWarps) {
    // ---------------- producer ----------------
    int s = 0, round = 0, n = 0;
    bool ok = true;
    for (int j = 0; j < S.nops && ok; ++j) {
      const StepOp& op = S.ops[j];
      int64_t ub, ue;
      step_units(op.a, cta, ub, ue);
      switch (op.fmt) {
        case FMT_NV4: ok = step_produce<FMT_NV4>(op.a, ub, ue, base, S.SLOT, S.NS, full0, empty0, s, round, n, S.err); break;
        case FMT_W6: ok = step_produce<FMT_W6>(op.a, ub, ue, base, S.SLOT, S.NS, full0, empty0, s, round, n, S.err); break;
        case FMT_MX8: ok = step_produce<FMT_MX8>(op.a, ub, ue, base, S.SLOT, S.NS, full0, empty0, s, round, n, S.err); break;
        default: ok = step_produce<FMT_W8>(op.a, ub, ue, base, S.SLOT, S.NS, full0, empty0, s, round, n, S.err); break;
      }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    // the number of stages issued, marked final (negative) for consumers that stopped early and drain the ring
    if ((threadIdx.x & 31) == 0) *reinterpret_cast<volatile int*>(issued) = -1 - n;
    return;
  }

  // ---------------- consumers ----------------
  pdl_wait();  // the first ops read what the previous kernel of the stream wrote
  StepConsumerState st{0, 0u, 0u, 0u, 0};
  int* stop = reinterpret_cast<int*>(base + S.smem_misc + 72);
  bool stopped = false;
  for (int j = 0; j < S.nops; ++j) {
    const StepOp& op = S.ops[j];
    int64_t ub, ue;
    step_units(op.a, cta, ub, ue);
    if (j == S.nops - 1) pdl_launch_dependents();
    step_stamp(S, j, 0);
    if (ue > ub) {
      // a warp whose bounded wait gave up has set the error word; every warp still reaches the barriers below
      switch (op.epi * 8 + op.fmt) {
        case EPI_STORE * 8 + FMT_NV4:
          step_consume<FMT_NV4, EPI_STORE>(S, op, (int)ub, (int)ue, base, full0, empty0, comb_full0,
                                                            comb_empty0, st);
          break;
        case EPI_STORE * 8 + FMT_W6:
          step_consume<FMT_W6, EPI_STORE>(S, op, (int)ub, (int)ue, base, full0, empty0, comb_full0,
                                                           comb_empty0, st);
          break;
        case EPI_STORE * 8 + FMT_MX8:
          step_consume<FMT_MX8, EPI_STORE>(S, op, (int)ub, (int)ue, base, full0, empty0, comb_full0,
                                                            comb_empty0, st);
          break;
        case EPI_HC_DOWN * 8 + FMT_W8:
          step_consume<FMT_W8, EPI_HC_DOWN>(S, op, (int)ub, (int)ue, base, full0, empty0, comb_full0,
                                                             comb_empty0, st);
          break;
        case EPI_HC_UP * 8 + FMT_W8:
          step_consume<FMT_W8, EPI_HC_UP>(S, op, (int)ub, (int)ue, base, full0, empty0, comb_full0,
                                                           comb_empty0, st);
          break;
        default:
          step_consume<FMT_W8, EPI_STORE>(S, op, (int)ub, (int)ue, base, full0, empty0, comb_full0,
                                                           comb_empty0, st);
          break;
      }
    }
    // the op is finished on this CTA once every consumer warp is past its last flush; one decision for all warps
    named_bar(1, kCWarps * 32);
    if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(stop) = ld_volatile(S.err) != 0;
    named_bar(1, kCWarps * 32);
    if (*reinterpret_cast<volatile int*>(stop)) {
      stopped = true;
      break;
    }
    if (threadIdx.x == 0) {
      __threadfence();
      atomicAdd(S.done + j, 1);
    }
    step_stamp(S, j, 3);
  }
  if (stopped) {
    // leave no bulk copy in flight: once the producer has stopped (it notices the error word), wait (bounded) for
    // every stage it issued that this warp has not taken
    const uint64_t t0 = global_ns();
    while (*reinterpret_cast<volatile int*>(issued) >= 0 && global_ns() - t0 < 2000000000ull) __nanosleep(1000);
    const int total = *reinterpret_cast<volatile int*>(issued);
    const int n = total >= 0 ? total : -1 - total;
    for (int i = st.consumed; i < n; ++i) {
      if (!mbar_wait_bounded(full0 + 8 * st.s, st.phase, nullptr, 2000000000ull)) break;
      if (++st.s == S.NS) { st.s = 0; st.phase ^= 1u; }
    }
    return;
  }
  // the last CTA to finish the step zeroes the counters for the next launch
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(S.fin, 1) == G - 1) {
      __threadfence();
      for (int j = 0; j < S.nops; ++j) S.done[j] = 0;
      *S.fin = 0;
      __threadfence();
    }
  }
}

}  // namespace fp4x
