// Host side of the persistent decode-step kernel (fp4x_step.cuh): per-op plans for one CTA per SM, the hazard
// analysis that orders the ops, the device op table, and the launch.
#include <algorithm>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "fp4x_launch.cuh"
#include "fp4x_step.cuh"

namespace fp4x {
namespace {

constexpr int kStepSlot = kStepSlotBytes;
constexpr int kStepWsRegions = 8;      // ops use workspace / semaphore regions round-robin
constexpr int kStepMisc = 512;

struct Range {
  uintptr_t lo, hi;
  bool overlaps(const Range& o) const { return lo < o.hi && o.lo < hi && hi > lo && o.hi > o.lo; }
};

struct OpInfo {
  StepOp op;
  std::vector<Range> reads, writes;
  int xp_max;  // largest staged activation pitch of any CTA (bytes per token)
  int kloc_max;  // largest staged k range of any CTA
};

struct StepLaunch {
  StepArgs args;
  int grid;
  int smem;
  int nt;
  int dev;
};

std::mutex g_step_mu;
std::unordered_map<const void*, StepLaunch> g_steps;

int esize(int dtype) { return dtype == FP4X_F32 ? 4 : 2; }

Range rows_range(const void* p, int64_t rows, int64_t stride, int64_t cols, int es) {
  const uintptr_t a = (uintptr_t)p;
  return Range{a, a + (uintptr_t)(((rows - 1) * stride + cols) * es)};
}

// per-kind geometry: format, epilogue, stage shape and the k per stage
struct KindGeom {
  int fmt, epi, shape, KC, BI0, NB0;
};
bool kind_geom(int kind, KindGeom& g) {
  switch (kind) {
    case FP4X_STEP_NV4: g = {FMT_NV4, EPI_STORE, SHAPE_128x2, 512, 128, 2}; return true;
    case FP4X_STEP_W6: g = {FMT_W6, EPI_STORE, SHAPE_128x1, 256, 128, 1}; return true;
    case FP4X_STEP_W8: g = {FMT_W8, EPI_STORE, SHAPE_128x2, 256, 128, 2}; return true;
    case FP4X_STEP_HC_DOWN: g = {FMT_W8, EPI_HC_DOWN, SHAPE_128x2, 256, 128, 2}; return true;
    case FP4X_STEP_HC_UP: g = {FMT_W8, EPI_HC_UP, SHAPE_128x2, 256, 128, 2}; return true;
    case FP4X_STEP_MX8: g = {FMT_MX8, EPI_STORE, SHAPE_128x2, 256, 128, 2}; return true;
  }
  return false;
}

int plan_op(const fp4x_step_op& o, int64_t m, int sms, int index, OpInfo& info) {
  const std::string where = "step op " + std::to_string(index) + ": ";
  KindGeom kg;
  if (!kind_geom(o.kind, kg)) return fail(FP4X_ERR_INVALID_ARG, where + "unknown kind");
  const FmtGeom G = fmt_geom(kg.fmt);
  const int64_t n = o.n, k = o.k;
  if (n < 1 || k < 1) return fail(FP4X_ERR_INVALID_ARG, where + "empty shape");
  if (k % kg.KC) return fail(FP4X_ERR_UNSUPPORTED, where + "K must be a multiple of " + std::to_string(kg.KC));
  if (!o.x || !o.p0 || (G.n1 && !o.p1) || !o.s) return fail(FP4X_ERR_INVALID_ARG, where + "null pointer");
  if (!aligned(o.x, 16) || o.x_stride % 8 || o.x_stride < k)
    return fail(FP4X_ERR_UNSUPPORTED, where + "activation rows must be 16-byte aligned");
  GemvArgs& a = info.op.a;
  std::memset(&info.op, 0, sizeof(info.op));
  info.op.fmt = kg.fmt;
  info.op.epi = kg.epi;
  info.op.shape = kg.shape;
  a.M = (int)m;
  a.N = (int)n;
  a.K = (int)k;
  a.x_stride = o.x_stride;
  a.KPW = (int)k;
  a.KP = 1;
  a.KC = kg.KC;
  a.NCH = (int)(k / kg.KC);
  a.RT = (int)((n + kRB - 1) / kRB);
  a.whole = kg.epi == EPI_HC_UP ? 1 : 0;
  {
    const int64_t units = a.whole ? a.RT : (int64_t)a.RT * a.NCH;
    a.CPP = (int)std::min<int64_t>(sms, units);  // every working CTA owns at least one unit
  }
  a.BI0 = kg.BI0;
  a.NB0 = kg.NB0;
  a.BI1 = G.n1 ? kg.KC * G.n1 / G.d1 : 0;
  a.SB = kg.KC * G.sn / G.sd;
  a.off_p1 = kRB * kg.NB0 * kg.BI0;
  a.off_sc = a.off_p1 + kRB * a.BI1;
  const int stg = (a.off_sc + kRB * a.SB + 1023) / 1024 * 1024;
  if (stg > kStepSlot) return fail(FP4X_ERR_UNSUPPORTED, where + "stage larger than the ring slot");
  a.STG = kStepSlot;
  a.group = 16;
  a.post = kg.fmt == FMT_NV4 ? o.gs : 1.f;
  a.xdirect = 1;
  const int64_t ld0 = k * G.n0 / G.d0, ld1 = G.n1 ? k * G.n1 / G.d1 : 0;
  a.lds = k * G.sn / G.sd;
  int rc;
  if (!aligned(o.p0, 16) || ld0 % 16) return fail(FP4X_ERR_UNSUPPORTED, where + "weight rows must be 16-byte aligned");
  if ((rc = encode_rows(&a.tm0, o.p0, n, ld0, kg.BI0))) return rc;
  if (G.n1) {
    if (!aligned(o.p1, 16) || ld1 % 16) return fail(FP4X_ERR_UNSUPPORTED, where + "plane-1 rows must be 16-byte aligned");
    if ((rc = encode_rows(&a.tm1, o.p1, n, ld1, a.BI1))) return rc;
  }
  a.scw = 0;
  for (int w : {16, 8, 4})
    if (a.SB % w == 0 && a.lds % w == 0 && aligned(o.s, w)) { a.scw = w; break; }
  if (!a.scw) return fail(FP4X_ERR_UNSUPPORTED, where + "scale rows must be 4-byte aligned");
  a.item = GemvItem{o.x, (const uint8_t*)o.s, o.out, o.out2};
  a.out_dtype = o.out_dtype;
  a.out_stride = o.out_stride;
  if (!o.out) return fail(FP4X_ERR_INVALID_ARG, where + "null output");
  // hazards: what the op reads and writes
  info.reads.push_back(rows_range(o.x, m, o.x_stride, k, 2));
  if (kg.epi == EPI_STORE) {
    if (o.out_stride < n) return fail(FP4X_ERR_INVALID_ARG, where + "out_stride < n");
    if (o.out_dtype < 0 || o.out_dtype > 2) return fail(FP4X_ERR_INVALID_ARG, where + "bad out_dtype");
    info.writes.push_back(rows_range(o.out, m, o.out_stride, n, esize(o.out_dtype)));
  } else if (kg.epi == EPI_HC_DOWN) {
    if (!o.out2 || o.lr < 1 || o.lr > n || o.hc < 1 || o.hc > 8) return fail(FP4X_ERR_INVALID_ARG, where + "bad lr/hc");
    a.lr = (int)o.lr;
    a.hc = (int)o.hc;
    a.out_stride = n;
    a.out_dtype = FP4X_BF16;
    info.writes.push_back(rows_range(o.out, m, n, n, 2));
    info.writes.push_back(rows_range(o.out2, m, o.lr, o.lr, 2));
  } else {  // EPI_HC_UP
    if (!o.nrm || o.hc < 1 || o.hc > 8 || o.bj < 1 || (o.hc * o.bj != 16 && o.hc * o.bj != 32) || n % (o.hc * o.bj) ||
        n % kRB)
      return fail(FP4X_ERR_UNSUPPORTED, where + "hc * bj must be 16 or 32 and the rows a multiple of 64");
    a.hc = (int)o.hc;
    a.bj = (int)o.bj;
    a.nrm = o.nrm;
    a.nrm_stride = o.nrm_stride;
    a.out_stride = n / o.hc;
    a.out_dtype = FP4X_BF16;
    info.reads.push_back(rows_range(o.nrm, m, o.nrm_stride, n, 2));
    info.writes.push_back(rows_range(o.out, m, n / o.hc, n / o.hc, 2));
  }
  // largest staged k range of any CTA (partial staging: only the chunks of the CTA's units)
  const int64_t Up = a.whole ? a.RT : (int64_t)a.RT * a.NCH;
  int nc_max = 0;
  for (int c = 0; c < a.CPP; ++c) {
    int64_t ub = range_begin(Up, a.CPP, c), ue = range_begin(Up, a.CPP, c + 1);
    if (a.whole) { ub *= a.NCH; ue *= a.NCH; }
    const int64_t nu = ue - ub;
    if (nu <= 0) continue;
    const int nc = (a.whole || nu >= a.NCH) ? a.NCH : (int)nu;
    nc_max = std::max(nc_max, nc);
  }
  info.xp_max = nc_max * (kg.KC / 16) * 32 + 32;
  info.kloc_max = nc_max * kg.KC;
  return FP4X_OK;
}

// dependencies: every earlier op with a read/write hazard, plus the op that last used the same scratch region;
// reduced to the ops not already implied by another dependency
int find_deps(std::vector<OpInfo>& ops, bool serial) {
  const int n = (int)ops.size();
  std::vector<std::vector<uint64_t>> anc(n, std::vector<uint64_t>((n + 63) / 64, 0));
  auto set_bit = [](std::vector<uint64_t>& v, int i) { v[i >> 6] |= 1ull << (i & 63); };
  auto has = [](const std::vector<uint64_t>& v, int i) { return (v[i >> 6] >> (i & 63)) & 1ull; };
  for (int j = 0; j < n; ++j) {
    std::vector<int> cand;
    for (int i = 0; i < j; ++i) {
      bool hz = (j - i) % kStepWsRegions == 0 || (serial && i == j - 1);
      for (const Range& w : ops[i].writes) {
        for (const Range& r : ops[j].reads) hz = hz || w.overlaps(r);
        for (const Range& w2 : ops[j].writes) hz = hz || w.overlaps(w2);
      }
      for (const Range& r : ops[i].reads)
        for (const Range& w : ops[j].writes) hz = hz || r.overlaps(w);
      if (hz) cand.push_back(i);
    }
    std::vector<int> keep;
    for (int i : cand) {
      bool implied = false;
      for (int i2 : cand)
        if (i2 != i && has(anc[i2], i)) { implied = true; break; }
      if (!implied) keep.push_back(i);
    }
    if ((int)keep.size() > kStepMaxDeps)
      return fail(FP4X_ERR_UNSUPPORTED, "step op " + std::to_string(j) + " depends on more than " +
                                            std::to_string(kStepMaxDeps) + " unrelated earlier ops");
    ops[j].op.ndeps = (int)keep.size();
    for (size_t d = 0; d < keep.size(); ++d) ops[j].op.deps[d] = keep[d];
    for (int i : cand) {
      set_bit(anc[j], i);
      for (size_t w = 0; w < anc[j].size(); ++w) anc[j][w] |= anc[i][w];
    }
  }
  return FP4X_OK;
}

struct StepSizes {
  size_t table, ws_region, ws;
  int64_t sem_region, counters;
  int xbytes, xraw, smem, ns;
};

int step_sizes(const std::vector<OpInfo>& ops, int64_t m, StepSizes& z) {
  const DeviceFacts& dv = device_facts();
  int xp = 0, rt = 1, kl = 0;
  for (const OpInfo& o : ops) {
    xp = std::max(xp, o.xp_max);
    kl = std::max(kl, o.kloc_max);
    rt = std::max(rt, o.op.a.RT);
  }
  z.table = ops.size() * sizeof(StepOp);
  const size_t slot = (size_t)kRW * 16 * 8 * sizeof(float);  // one warp's 16 x 8 partial tile
  z.ws_region = (size_t)dv.sms * 2 * slot;
  z.ws = z.ws_region * kStepWsRegions;
  z.sem_region = (int64_t)rt * kRW;
  z.counters = (int64_t)ops.size() + 1 + z.sem_region * kStepWsRegions;
  z.xbytes = (int)(((int64_t)m * xp + 15) / 16 * 16);
  z.xraw = (int)(((int64_t)m * kl * 2 + 15) / 16 * 16);
  const int scr = kRW * 16 * 8 * 4, comb = kRW * 32 * 4 * 4;
  const int fixed = z.xbytes + z.xraw + kStepMisc + scr + comb + 1024;
  int ns = (dv.smem_optin - fixed) / kStepSlot;
  if (ns > kStepMaxStages) ns = kStepMaxStages;
  if (ns < 3) return fail(FP4X_ERR_UNSUPPORTED, "step activations leave too little shared memory for the stage ring");
  z.ns = ns;
  z.smem = ns * kStepSlot + fixed;
  return FP4X_OK;
}

int build_ops(const fp4x_step_op* ops, int64_t count, int64_t m, bool serial, std::vector<OpInfo>& infos,
              StepSizes& z) {
  if (!ops || count < 1 || count > 4096) return fail(FP4X_ERR_INVALID_ARG, "bad op list");
  if (m < 1 || m > 8) return fail(FP4X_ERR_UNSUPPORTED, "the step kernel runs 1..8 tokens");
  const int sms = device_facts().sms;
  infos.resize((size_t)count);
  int rc;
  for (int64_t i = 0; i < count; ++i)
    if ((rc = plan_op(ops[i], m, sms, (int)i, infos[(size_t)i]))) return rc;
  if ((rc = find_deps(infos, serial))) return rc;
  return step_sizes(infos, m, z);
}

}  // namespace
}  // namespace fp4x

using namespace fp4x;

extern "C" {

int fp4x_step_query(const fp4x_step_op* ops, int64_t count, int64_t m, int serial, size_t* table_bytes,
                    size_t* ws_bytes, int64_t* n_counters) {
  std::vector<OpInfo> infos;
  StepSizes z;
  int rc = build_ops(ops, count, m, serial != 0, infos, z);
  if (rc) return rc;
  if (table_bytes) *table_bytes = z.table;
  if (ws_bytes) *ws_bytes = z.ws;
  if (n_counters) *n_counters = z.counters;
  return FP4X_OK;
}

int fp4x_step_prepare(const fp4x_step_op* ops, int64_t count, int64_t m, int serial, void* table, size_t table_bytes,
                      void* ws, size_t ws_bytes, int32_t* counters, int64_t n_counters) {
  std::vector<OpInfo> infos;
  StepSizes z;
  int rc = build_ops(ops, count, m, serial != 0, infos, z);
  if (rc) return rc;
  if (!table || table_bytes < z.table || !aligned(table, 64))
    return fail(FP4X_ERR_WORKSPACE, "op table too small or not 64-byte aligned (see fp4x_step_query)");
  if (!ws || ws_bytes < z.ws || !aligned(ws, 16) || !counters || n_counters < z.counters)
    return fail(FP4X_ERR_WORKSPACE, "step scratch too small (see fp4x_step_query)");
  int* done = counters;
  int* sem0 = counters + count + 1;
  std::vector<StepOp> host((size_t)count);
  for (int64_t j = 0; j < count; ++j) {
    StepOp& op = infos[(size_t)j].op;
    const int r = (int)(j % kStepWsRegions);
    op.a.ws = (float*)((uint8_t*)ws + (size_t)r * z.ws_region);
    op.a.sem = sem0 + (int64_t)r * z.sem_region;
    op.a.err = dev_error_ptr();
    op.a.NS = z.ns;
    host[(size_t)j] = op;
  }
  cudaError_t e = cudaMemcpy(table, host.data(), z.table, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return check_launch(e, "copying the step table");
  StepLaunch L;
  std::memset(&L, 0, sizeof(L));
  L.args.ops = (const StepOp*)table;
  L.args.nops = (int)count;
  L.args.NS = z.ns;
  L.args.SLOT = kStepSlot;
  L.args.smem_x = z.ns * kStepSlot;
  L.args.smem_xraw = L.args.smem_x + z.xbytes;
  L.args.smem_misc = L.args.smem_xraw + z.xraw;
  L.args.smem_scr = L.args.smem_misc + kStepMisc;
  L.args.smem_comb = L.args.smem_scr + kRW * 16 * 8 * 4;
  L.args.done = done;
  L.args.fin = counters + count;
  L.args.err = dev_error_ptr();
  L.grid = device_facts().sms;
  L.smem = z.smem;
  L.nt = 1;
  cudaGetDevice(&L.dev);
  std::lock_guard<std::mutex> lk(g_step_mu);
  g_steps[table] = L;
  return FP4X_OK;
}

int fp4x_step_run(const void* table, void* stream) {
  StepLaunch L;
  {
    std::lock_guard<std::mutex> lk(g_step_mu);
    auto it = g_steps.find(table);
    if (it == g_steps.end()) return fail(FP4X_ERR_INVALID_ARG, "step table was not prepared (fp4x_step_prepare)");
    L = it->second;
  }
  auto kern = step_kernel<1>;
  cudaError_t e = ensure_smem_attr((const void*)kern, L.smem);
  if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute(step)");
  e = launch_pdl(kern, dim3(L.grid), dim3(kThreads), (size_t)L.smem, (cudaStream_t)stream, L.args);
  if (e != cudaSuccess) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, (const void*)kern);
    return fail(FP4X_ERR_CUDA, std::string("step launch: ") + cudaGetErrorString(e) + " (registers " +
                                   std::to_string(fa.numRegs) + ", max threads " + std::to_string(fa.maxThreadsPerBlock) +
                                   ", local bytes " + std::to_string(fa.localSizeBytes) + ", shared " +
                                   std::to_string(L.smem) + " + static " + std::to_string(fa.sharedSizeBytes) + ")");
  }
  return FP4X_OK;
}

int fp4x_step_trace(const void* table, uint64_t* trace, int64_t entries) {
  std::lock_guard<std::mutex> lk(g_step_mu);
  auto it = g_steps.find(table);
  if (it == g_steps.end()) return fail(FP4X_ERR_INVALID_ARG, "unknown step table");
  if (trace && entries < (int64_t)it->second.grid * it->second.args.nops * 8)
    return fail(FP4X_ERR_WORKSPACE, "trace buffer needs grid * ops * 8 entries");
  it->second.args.trace = trace;
  return FP4X_OK;
}

int fp4x_step_release(const void* table) {
  std::lock_guard<std::mutex> lk(g_step_mu);
  return g_steps.erase(table) ? FP4X_OK : fail(FP4X_ERR_INVALID_ARG, "unknown step table");
}

}  // extern "C"
