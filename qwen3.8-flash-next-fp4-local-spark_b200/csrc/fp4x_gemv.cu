// Host planner, TMA descriptors, launchers and C ABI of the GEMV family (MXFP8, W8, W6, NVFP4, BF16, INT2, batched
// W8 and the fused / unfused hyper-connection mixer).
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "fp4x_gemv.cuh"
#include "fp4x_launch.cuh"
#include "fp4x_host.h"

namespace fp4x {

__device__ int g_dev_error = 0;
std::atomic<int64_t> g_launches{0};

// launch timeline (diagnostic): a device buffer of kTlWords words per launch, handed out in launch order
static std::atomic<unsigned long long*> g_tl_buf{nullptr};
static std::atomic<int64_t> g_tl_cap{0}, g_tl_next{0};

unsigned long long* timeline_next() {
  unsigned long long* b = g_tl_buf.load(std::memory_order_acquire);
  if (!b) return nullptr;
  const int64_t i = g_tl_next.fetch_add(1, std::memory_order_relaxed);
  return i < g_tl_cap.load(std::memory_order_relaxed) ? b + kTlWords * i : nullptr;
}

int* dev_error_ptr() {
  static int* ptrs[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev & 63]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_dev_error) == cudaSuccess) ptrs[dev & 63] = (int*)p;
  }
  return ptrs[dev & 63];
}

static thread_local std::string t_msg;
void set_error_message(const std::string& msg) { t_msg = msg; }
int fail(int code, const std::string& msg) {
  t_msg = msg;
  return code;
}

const DeviceFacts& device_facts() {
  static DeviceFacts facts[64];
  static bool have[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!have[dev & 63]) {
    DeviceFacts f{};
    cudaDeviceGetAttribute(&f.sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&f.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    cudaDeviceGetAttribute(&f.smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    if (f.sms <= 0) f.sms = 148;
    if (f.smem_optin <= 0) f.smem_optin = 227 * 1024;
    if (f.smem_sm <= 0) f.smem_sm = 228 * 1024;
    facts[dev & 63] = f;
    have[dev & 63] = true;
  }
  return facts[dev & 63];
}

cudaError_t ensure_smem_attr(const void* kernel, int bytes) {
  // remembers the largest value set per (kernel, device)
  struct Entry {
    const void* k;
    int dev;
    int bytes;
  };
  static Entry tab[512];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (tab[i].k == kernel && tab[i].dev == dev && tab[i].bytes >= bytes) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess && n < 512) tab[n++] = Entry{kernel, dev, bytes};
  return e;
}

// allow clusters of up to 16 CTAs for a kernel, once per (kernel, device)
cudaError_t ensure_nonportable_cluster(const void* kernel) {
  static const void* done_k[256];
  static int done_d[256];
  static int n = 0;
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n; ++i)
    if (done_k[i] == kernel && done_d[i] == dev) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e == cudaSuccess && n < 256) { done_k[n] = kernel; done_d[n] = dev; ++n; }
  return e;
}

// ------------------------------------------------------------------------------------------------------
// TMA descriptors: 2D [rows, row_bytes] uint8 views, box {inner, 64 rows}, 64B/128B swizzle; cached per device
// ------------------------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)p;
  });
  return fn;
}

static int encode_rows_uncached(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int inner) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FP4X_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t gdim[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)inner, (cuuint32_t)kRB};
  const cuuint32_t es[2] = {1, 1};
  const CUtensorMapSwizzle sw = inner == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), gdim, gstride, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FP4X_ERR_UNSUPPORTED, "tensor map encode failed (" + std::to_string((int)r) + ")");
  return FP4X_OK;
}

// [rows][row_bytes] u8 scale rows, box {box_bytes, 128 rows}, no swizzle (the tcgen05 kernels' scale tiles)
int encode_scale_box(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int box_bytes) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FP4X_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t gdim[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, 128};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), gdim, gstride, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FP4X_ERR_UNSUPPORTED, "scale tensor map encode failed (" + std::to_string((int)r) + ")");
  return FP4X_OK;
}

// [rows][row_bytes] u8, box {box_bytes, box_rows}, 64-byte swizzle when box_bytes is 64 (the INT2 code tiles)
int encode_box(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int box_bytes, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FP4X_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t gdim[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
  const cuuint64_t gstride[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)box_bytes, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUtensorMapSwizzle sw = box_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), gdim, gstride, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FP4X_ERR_UNSUPPORTED, "tensor map encode failed (" + std::to_string((int)r) + ")");
  return FP4X_OK;
}

int encode_rows(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int inner) {
  struct Key {
    uintptr_t p;
    int64_t rows, rb;
    int inner;
    bool operator==(const Key& o) const { return p == o.p && rows == o.rows && rb == o.rb && inner == o.inner; }
  };
  struct KeyHash {
    size_t operator()(const Key& k) const {
      return std::hash<uintptr_t>()(k.p) ^ (std::hash<int64_t>()(k.rows) * 31) ^ (std::hash<int64_t>()(k.rb) * 131) ^
             (size_t)k.inner;
    }
  };
  static std::unordered_map<Key, CUtensorMap, KeyHash> cache;
  static std::mutex mu;
  const Key key{(uintptr_t)ptr, rows, row_bytes, inner};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto itc = cache.find(key);
    if (itc != cache.end()) {
      *tm = itc->second;
      return FP4X_OK;
    }
  }
  int rc = encode_rows_uncached(tm, ptr, rows, row_bytes, inner);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 16384) cache.clear();
  cache.emplace(key, *tm);
  return FP4X_OK;
}

// ------------------------------------------------------------------------------------------------------
// planning
// ------------------------------------------------------------------------------------------------------
enum PlanMode { kStreamK = 0, kWholeTile = 1 };


static int round_up(int v, int a) { return (v + a - 1) / a * a; }

static double bytes_per_k(int fmt, int group) {
  const FmtGeom G = fmt_geom(fmt);
  double b = (double)G.n0 / G.d0 + (G.n1 ? (double)G.n1 / G.d1 : 0.0);
  if (G.sn) b += fmt == FMT_INT2 ? 2.0 / group : (double)G.sn / G.sd;
  return b;
}

// stage chunk for a panel: plane-0 bytes per row per stage 256 (two 128-byte boxes), 128 or 64 (one box)
static bool chunk_for(int fmt, int kpw, int& KC, int& BI0, int& NB0) {
  const FmtGeom G = fmt_geom(fmt);
  const int pbs[3] = {256, 128, 64};
  for (int pb : pbs) {
    const int kc = pb * G.d0 / G.n0;
    if (kc % G.kmin || kpw % kc) continue;
    if (fmt == FMT_W6 && pb < 128) continue;  // the high-bit plane needs >= 64-byte boxes
    if (fmt == FMT_MX8 && kc < 128) continue;  // scale rows of >= 4 bytes per stage
    KC = kc;
    BI0 = pb >= 128 ? 128 : 64;
    NB0 = pb / BI0;
    return true;
  }
  return false;
}

// Cluster plan: one row block per CTA, K split into KP panels (2..8) whose CTAs form a (1, KP, 1) cluster; the
// panel partials are summed in the leader's shared memory.  Picks the largest KP with RT * KP <= 2 * SMs whose panel
// width has a valid stage shape.  `base` carries the shape fields (NT, MP, RT).
static bool make_cluster_plan(int fmt, int64_t M, int64_t N, int64_t K, int group, const Plan& base, Plan& out) {
  const FmtGeom G = fmt_geom(fmt);
  const DeviceFacts& dv = device_facts();
  const int sd = fmt == FMT_INT2 ? group / 2 : G.sd;
  const int misc = 512;
  const int comb_bytes = kRW * 32 * base.NT * 4 * 4;
  for (int KP = 8; KP >= 2; --KP) {
    // at 16 tokens one CTA per SM (the 128-register entry: the two-per-SM stage bodies spill)
    if (K % KP || (int64_t)base.RT * KP > (base.NT == 2 ? 1 : 2) * dv.sms) continue;
    const int kpw = (int)(K / KP);
    int KC, BI0, NB0;
    if (kpw % 64 || !chunk_for(fmt, kpw, KC, BI0, NB0)) continue;
    if (fmt == FMT_W8 && BI0 == 64) continue;  // one 64-group per stage would leave a k-group idle
    Plan c = base;
    c.KPW = kpw; c.KP = KP; c.KC = KC; c.BI0 = BI0; c.NB0 = NB0; c.NCH = kpw / KC;
    c.BI1 = G.n1 ? KC * G.n1 / G.d1 : 0;
    c.SB = G.sn ? KC * G.sn / sd : 0;
    if (c.SB % 4) continue;
    c.off_p1 = kRB * NB0 * BI0;
    c.off_sc = c.off_p1 + kRB * c.BI1;
    c.STG = round_up(c.off_sc + kRB * c.SB, 1024);
    c.XP = (kpw / 16) * 32 + 32;
    const int red_bytes = (KP - 1) * kRW * 32 * c.NT * 16;
    c.xdirect = 0;
    const int raw = fmt == FMT_W8 ? 0 : (int)M * kpw * 2;  // W8 stages into the operand panel directly
    const int xbytes = round_up(c.MP * c.XP, 16) + raw;
    const int fixed = xbytes + misc + comb_bytes + red_bytes + 1024;
    const int ctas = base.RT * KP;
    const int cap = ctas > dv.sms ? dv.smem_sm / 2 - 2048 : dv.smem_optin;
    int ns = (cap - fixed) / c.STG;
    if (ns > kMaxStages) ns = kMaxStages;
    if (ns > c.NCH) ns = c.NCH;  // a CTA streams NCH stages in all
    if (ns < 1 || (c.NCH > 1 && ns < 2)) continue;
    c.NS = ns;
    c.CPP = base.RT;
    c.whole = 1;
    c.SMAX = 1;
    c.smem_x = c.NS * c.STG;
    c.smem_misc = c.smem_x + round_up(c.MP * c.XP, 16);
    c.smem_scr = c.smem_misc + misc;
    c.smem_xraw = c.smem_scr;
    c.smem_comb = c.smem_xraw + round_up(raw, 16);
    c.smem_red = c.smem_comb + comb_bytes;
    c.smem_total = c.smem_red + red_bytes + 1024;
    c.ws_bytes = 0;
    c.counters = 0;
    c.cluster = KP;
    out = c;
    return true;
  }
  return false;
}

// returns 0 and fills `pl`, or a negative status
static int make_plan(int fmt, int64_t M, int64_t N, int64_t K, int64_t batch, int group, PlanMode mode,
                     int epi_scratch, Plan& pl) {
  if (M < 1 || M > 16) return fail(FP4X_ERR_INVALID_ARG, "M must be in 1..16 (decode shapes)");
  if (N < 1 || K < 1 || batch < 1) return fail(FP4X_ERR_INVALID_ARG, "empty shape");
  if (N > (1 << 30) || K > (1 << 20)) return fail(FP4X_ERR_UNSUPPORTED, "shape too large");
  const FmtGeom G = fmt_geom(fmt);
  if (fmt == FMT_INT2 && group != 16 && group != 32) return fail(FP4X_ERR_UNSUPPORTED, "INT2 group must be 16 or 32");
  const int kmin = fmt == FMT_MX8 ? 128 : G.kmin;
  if (K % 64 != 0 || K % kmin != 0)
    return fail(FP4X_ERR_UNSUPPORTED, "K=" + std::to_string(K) + " must be a multiple of " + std::to_string(kmin > 64 ? kmin : 64));
  const DeviceFacts& dv = device_facts();
  pl.NT = M <= 8 ? 1 : 2;
  pl.MP = 8 * pl.NT;
  pl.RT = (int)((N + kRB - 1) / kRB);
  // INT2 heads always use whole row blocks: each row's fp32 sum then has a fixed order that does not depend on the
  // vocabulary size or the grid, so a vocab-sharded head reproduces the unsharded coarse values bit for bit
  const bool whole = (mode == kWholeTile || fmt == FMT_INT2);
  pl.whole = whole ? 1 : 0;
  const int sd = fmt == FMT_INT2 ? group / 2 : G.sd;
  const double wbytes = (double)batch * N * K * bytes_per_k(fmt, group);
  const int misc = 512;
  const int scr_bytes = epi_scratch ? kRW * 16 * pl.MP * 4 : 0;
  const int comb_bytes = kRW * 32 * pl.NT * 4 * 4;
  const int cap1 = dv.smem_optin;
  const int cap2 = dv.smem_sm / 2 - 2048;  // two CTAs per SM (1 KB reserved per CTA, 1 KB alignment slack)

  // 16-token plans: the raw activation panel (M x panel x 2 bytes) may stay in global memory (staging then reads
  // it from L2) when keeping it in shared memory would force the K dimension into more than two panels.
  bool found = false;
  Plan best = pl;
  for (int direct = 0; direct <= (pl.NT == 2 ? 1 : 0); ++direct) {
  if (direct && found && best.KP <= 2) break;
  bool found_d = false;
  double best_score = -1e30;
  Plan best_d = pl;
  for (int kpw = (int)K; kpw >= 64; --kpw) {
    if (K % kpw) continue;
    if (whole && kpw != K) break;
    int KC, BI0, NB0;
    if (!chunk_for(fmt, kpw, KC, BI0, NB0)) continue;
    Plan c = pl;
    c.KPW = kpw;
    c.KP = (int)(K / kpw);
    c.KC = KC;
    c.BI0 = BI0;
    c.NB0 = NB0;
    c.NCH = kpw / KC;
    c.BI1 = G.n1 ? KC * G.n1 / G.d1 : 0;
    c.SB = G.sn ? KC * G.sn / sd : 0;
    if (c.SB % 4) continue;
    c.off_p1 = kRB * NB0 * BI0;
    c.off_sc = c.off_p1 + kRB * c.BI1;
    c.STG = round_up(c.off_sc + kRB * c.SB, 1024);
    c.XP = (kpw / 16) * 32 + 32;
    c.xdirect = direct;
    // operand panel + raw panel (W8 copies the rows straight into the operand panel: no raw panel)
    const int xbytes = round_up(c.MP * c.XP, 16) + (c.xdirect || fmt == FMT_W8 ? 0 : (int)M * kpw * 2);
    const int fixed = xbytes + misc + scr_bytes + comb_bytes + 1024;
    // 16-token stream-K plans keep one CTA per SM (the 128-register entry): at two per SM their stage bodies spill
    // (the 48 router gates at M = 16: 46 against 62 µs).  Whole-tile plans (HC up) keep the choice: with more row
    // blocks than SMs, one CTA per SM leaves some SMs two blocks in a row (the mixer at M = 16: 20.4 against 18.2 µs).
    for (int cps = (pl.NT == 2 && !whole) ? 1 : 2; cps >= 1; --cps) {
      const int cap = cps == 2 ? cap2 : cap1;
      int ns = (cap - fixed) / c.STG;
      if (ns > kMaxStages) ns = kMaxStages;
      if (ns < 2 || (cps == 2 && ns < 3)) continue;
      const double inflight = (double)cps * ns * c.STG;
      const int ctas = cps * dv.sms;
      const double share = wbytes / ctas;
      // score: bytes in flight per SM (up to ~128 KB), minus the relative cost of staging activations per CTA and of
      // the cross-panel reduction traffic.  Batched launches (many small matrices) take two CTAs per SM when they can:
      // measured on the 48 router gates, 29 µs against 42 µs with one wide CTA per SM at M = 4..8.
      const double x_cost = (double)c.MP * kpw * 2 / (share > 1 ? share : 1);
      const double red_cost = c.KP > 1 ? (double)c.KP * N * c.MP * 8.0 * batch / wbytes : 0.0;
      const double score = (inflight < 131072 ? inflight : 131072) / 131072.0 - 0.5 * x_cost - red_cost +
                           (batch > 1 && cps == 2 ? 0.5 : 0.0);
      if (score > best_score) {
        best_score = score;
        c.NS = ns;
        c.CPP = cps;  // CTAs per SM for now
        best_d = c;
        found_d = true;
      }
      break;
    }
  }
  if (found_d && (!found || best_d.KP < best.KP)) {
    best = best_d;
    found = true;
  }
  }
  if (!found) return fail(FP4X_ERR_UNSUPPORTED, "shape needs more shared memory than available");
  pl = best;
  const int cps = pl.CPP;
  const int64_t Up = whole ? (int64_t)pl.RT : (int64_t)pl.RT * pl.NCH;
  int64_t cpp = (int64_t)cps * dv.sms / (pl.KP * batch);
  if (cpp < 1) cpp = 1;
  if (cpp > Up) cpp = Up;  // every CTA owns at least one unit
  pl.CPP = (int)cpp;
  pl.smem_x = pl.NS * pl.STG;
  pl.smem_misc = pl.smem_x + round_up(pl.MP * pl.XP, 16);
  pl.smem_scr = pl.smem_misc + misc;
  pl.smem_xraw = pl.smem_scr + round_up(scr_bytes, 16);
  pl.smem_comb = pl.smem_xraw + round_up(pl.xdirect || fmt == FMT_W8 ? 0 : (int)M * pl.KPW * 2, 16);
  pl.smem_total = pl.smem_comb + comb_bytes + 1024;
  pl.SMAX = whole ? 1 : (int)((int64_t)(pl.NCH - 1) * pl.CPP / Up) + 2;
  if (pl.SMAX > pl.CPP) pl.SMAX = pl.CPP;
  const size_t slot = (size_t)kRW * 16 * pl.MP * sizeof(float);
  const bool split = !whole && pl.NCH > 1;
  if (pl.KP > 1)
    pl.ws_bytes = (size_t)batch * pl.KP * pl.RT * pl.SMAX * slot;
  else if (split)
    pl.ws_bytes = (size_t)batch * pl.CPP * 2 * slot;
  else
    pl.ws_bytes = 0;
  pl.counters = (pl.KP > 1 || split) ? (int64_t)batch * pl.RT * kRW : 0;
  pl.cluster = 0;
  pl.smem_red = pl.smem_total;
  // Small row counts: split K into panels whose CTAs form one cluster per row block and reduce on chip.
  if (mode == kStreamK && !whole && batch == 1 && fmt != FMT_INT2 && 2 * pl.RT <= dv.sms) {
    Plan cp;
    if (make_cluster_plan(fmt, M, N, K, group, pl, cp)) pl = cp;
  }
  return FP4X_OK;
}

// ------------------------------------------------------------------------------------------------------
// launch
// ------------------------------------------------------------------------------------------------------
static void fill_args(const Plan& pl, GemvArgs& a) {
  a.err = dev_error_ptr();
  a.tl = timeline_next();
  a.KPW = pl.KPW; a.KP = pl.KP; a.KC = pl.KC; a.NCH = pl.NCH; a.CPP = pl.CPP; a.RT = pl.RT; a.NS = pl.NS;
  a.SMAX = pl.SMAX; a.whole = pl.whole;
  a.BI0 = pl.BI0; a.BI1 = pl.BI1; a.NB0 = pl.NB0; a.SB = pl.SB; a.STG = pl.STG;
  a.off_p1 = pl.off_p1; a.off_sc = pl.off_sc; a.XP = pl.XP;
  a.smem_x = pl.smem_x; a.smem_misc = pl.smem_misc; a.smem_scr = pl.smem_scr; a.smem_xraw = pl.smem_xraw;
  a.xdirect = pl.xdirect;
  a.smem_comb = pl.smem_comb;
  a.cluster = pl.cluster; a.smem_red = pl.smem_red;
}

// widest cp.async (16/8/4 bytes) that keeps every scale copy aligned
static int scale_width(const void* sc, int64_t lds, int SB) {
  for (int w : {16, 8, 4})
    if (SB % w == 0 && lds % w == 0 && aligned(sc, w)) return w;
  return 0;
}

static int check_scratch(const Plan& pl, void* ws, size_t ws_bytes, int32_t* counters, int64_t n_counters) {
  if (pl.ws_bytes && (ws == nullptr || ws_bytes < pl.ws_bytes))
    return fail(FP4X_ERR_WORKSPACE, "workspace too small: need " + std::to_string(pl.ws_bytes) + " bytes");
  if (pl.counters && (counters == nullptr || n_counters < pl.counters))
    return fail(FP4X_ERR_WORKSPACE, "counter array too small: need " + std::to_string(pl.counters));
  if (ws && !aligned(ws, 16)) return fail(FP4X_ERR_UNSUPPORTED, "workspace must be 16-byte aligned");
  return FP4X_OK;
}

static int check_x(const void* x, int64_t x_stride, int64_t K) {
  if (!x) return fail(FP4X_ERR_INVALID_ARG, "null activation pointer");
  if (!aligned(x, 16) || x_stride % 8 != 0 || x_stride < K)
    return fail(FP4X_ERR_UNSUPPORTED, "activation rows must be 16-byte aligned (stride multiple of 8 elements)");
  return FP4X_OK;
}

static int check_out_dtype(int d) {
  if (d != FP4X_BF16 && d != FP4X_F16 && d != FP4X_F32) return fail(FP4X_ERR_INVALID_ARG, "bad out_dtype");
  return FP4X_OK;
}

static int check_rows(const void* p, int64_t row_bytes, const char* what) {
  if (!p) return fail(FP4X_ERR_INVALID_ARG, std::string("null ") + what);
  if (!aligned(p, 16) || row_bytes % 16 != 0)
    return fail(FP4X_ERR_UNSUPPORTED, std::string(what) + " rows must be 16-byte aligned");
  return FP4X_OK;
}

// shared path of the single-matrix GEMVs
static int run_gemv(int fmt, const void* x, int64_t x_stride, const void* p0, const void* p1, const void* sc,
                    float post, int group, void* out, void* out2, int64_t out_stride, int out_dtype, int64_t m,
                    int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters, int64_t n_counters,
                    void* stream, int epi, PlanMode mode = kStreamK, int lr = 0, int hc = 0) {
  int rc;
  if ((rc = check_out_dtype(out_dtype))) return rc;
  Plan pl;
  if ((rc = make_plan(fmt, m, n, k, 1, group, mode, 0, pl))) return rc;
  if ((rc = check_x(x, x_stride, k))) return rc;
  const FmtGeom G = fmt_geom(fmt);
  const int64_t ld0 = k * G.n0 / G.d0, ld1 = G.n1 ? k * G.n1 / G.d1 : 0;
  const int sd = fmt == FMT_INT2 ? group / 2 : G.sd;
  const int64_t lds = G.sn ? k * G.sn / sd : 0;
  if ((rc = check_rows(p0, ld0, "weight"))) return rc;
  if (G.n1 && (rc = check_rows(p1, ld1, "weight plane 1"))) return rc;
  int scw = 0;
  if (G.sn) {
    if (!sc) return fail(FP4X_ERR_INVALID_ARG, "null scales");
    scw = scale_width(sc, lds, pl.SB);
    if (!scw) return fail(FP4X_ERR_UNSUPPORTED, "scale rows must be 4-byte aligned");
  }
  if (!out) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (out_stride < n) return fail(FP4X_ERR_INVALID_ARG, "out_stride < n");
  if ((rc = check_scratch(pl, ws, ws_bytes, counters, n_counters))) return rc;
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  if ((rc = encode_rows(&a.tm0, p0, n, ld0, pl.BI0))) return rc;
  if (G.n1 && (rc = encode_rows(&a.tm1, p1, n, ld1, pl.BI1))) return rc;
  a.item = GemvItem{x, (const uint8_t*)sc, out, out2};
  a.batch = nullptr;
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = x_stride; a.lds = lds; a.scw = scw;
  a.out_stride = out_stride; a.out_dtype = out_dtype; a.post = post; a.group = group;
  a.lr = lr; a.hc = hc;
  a.ws = (float*)ws; a.sem = counters;
  fill_args(pl, a);
  cudaStream_t st = (cudaStream_t)stream;
  switch (fmt) {
    case FMT_MX8: return launch_nt<FMT_MX8, EPI_STORE>(pl, a, 1, st);
    case FMT_W8:
      if (epi == EPI_HC_DOWN) return launch_nt<FMT_W8, EPI_HC_DOWN>(pl, a, 1, st);
      return launch_nt<FMT_W8, EPI_STORE>(pl, a, 1, st);
    case FMT_W6: return launch_nt<FMT_W6, EPI_STORE>(pl, a, 1, st);
    case FMT_NV4: return launch_nt<FMT_NV4, EPI_STORE>(pl, a, 1, st);
    case FMT_BF16: return launch_nt<FMT_BF16, EPI_STORE>(pl, a, 1, st);
    case FMT_INT2: return launch_nt<FMT_INT2, EPI_HEAD>(pl, a, 1, st);
  }
  return fail(FP4X_ERR_INVALID_ARG, "bad format");
}

// ------------------------------------------------------------------------------------------------------
// small elementwise kernels of the unfused mixer route
// ------------------------------------------------------------------------------------------------------
__global__ void hc_scaled_silu_kernel(const __nv_bfloat16* di, __nv_bfloat16* bot, int M, int N, int lr, int hc) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M * lr; i += gridDim.x * blockDim.x) {
    const int m = i / lr, n = i - m * lr;
    const float t = bf16_round(__bfloat162float(di[(int64_t)m * N + n]) / (float)hc);
    bot[i] = __float2bfloat16_rn(t * sigmoidf_(t));
  }
}

__global__ void hc_gate_mean_kernel(const __nv_bfloat16* g, const __nv_bfloat16* nrm, int64_t nrm_stride,
                                    __nv_bfloat16* out, int M, int H, int hc) {
  pdl_wait();
  pdl_launch_dependents();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M * H; i += gridDim.x * blockDim.x) {
    const int m = i / H, j = i - m * H;
    float nv[8], gv[8];
    for (int s = 0; s < hc; ++s) {
      nv[s] = __bfloat162float(nrm[(int64_t)m * nrm_stride + s * H + j]);
      gv[s] = bf16_round(sigmoidf_(__bfloat162float(g[(int64_t)m * hc * H + s * H + j])));
    }
    out[(int64_t)m * H + j] = __float2bfloat16_rn(hc_gate_mean(nv, gv, hc));
  }
}

// Test hook of the bounded waits: one CTA waits on an mbarrier that no thread arrives on, through the production
// wait with a short limit; the wait gives up, records kDevWaitTimeout in the error word and the kernel returns.
__global__ void expire_wait_kernel(int* err, uint64_t limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    mbar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait_bounded(smem_u32(&bar), 0, err, limit_ns);
}

int reset_static_counters(cudaStream_t st);

}  // namespace fp4x

using namespace fp4x;

// ------------------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------------------
extern "C" {

int fp4x_version(void) { return 200; }

const char* fp4x_last_error_message(void) { return t_msg.c_str(); }

int64_t fp4x_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int fp4x_timeline_begin(void* records, int64_t count) {
#ifndef FP4X_TIMELINE
  (void)records;
  (void)count;
  return fail(FP4X_ERR_UNSUPPORTED, "built without FP4X_TIMELINE: the timeline is in libfp4x_timeline.so");
#endif
  if (!records || count < 1) return fail(FP4X_ERR_INVALID_ARG, "timeline needs a buffer of count >= 1 records");
  g_tl_cap.store(count, std::memory_order_relaxed);
  g_tl_next.store(0, std::memory_order_relaxed);
  g_tl_buf.store((unsigned long long*)records, std::memory_order_release);
  return FP4X_OK;
}

int64_t fp4x_timeline_end(void) {
  g_tl_buf.store(nullptr, std::memory_order_release);
  const int64_t n = g_tl_next.load(std::memory_order_relaxed), cap = g_tl_cap.load(std::memory_order_relaxed);
  return n < cap ? n : cap;
}

int fp4x_device_error(void* stream, int clear, int* code_out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, std::string("reading the device error word: ") + cudaGetErrorString(e));
  if (code_out) *code_out = v;
  if (clear && v) {
    // a kernel that gave up may have left arrival counters mid-count: the library's own static counters are
    // zeroed here (caller-owned counter arrays are the caller's to zero)
    int rc = reset_static_counters((cudaStream_t)stream);
    if (rc) return rc;
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, cudaGetErrorString(e));
  }
  return v ? fail(FP4X_ERR_DEVICE, "device error word = " + std::to_string(v)) : FP4X_OK;
}

int fp4x_test_expire_wait(int64_t limit_ns, void* stream) {
  if (limit_ns < 1000 || limit_ns > 1000000000) return fail(FP4X_ERR_INVALID_ARG, "limit_ns must be in [1e3, 1e9]");
  int* err = dev_error_ptr();
  if (!err) return fail(FP4X_ERR_CUDA, "device error word not available");
  expire_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(err, (uint64_t)limit_ns);
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return check_launch(cudaGetLastError(), "expire-wait test kernel");
}

int fp4x_gemv_query(int fmt, int64_t m, int64_t n, int64_t k, int64_t batch, int group, size_t* ws_bytes,
                    int64_t* n_counters) {
  if (fmt < 0 || fmt > 5) return fail(FP4X_ERR_INVALID_ARG, "bad format");
  Plan pl;
  int rc = make_plan(fmt, m, n, k, batch, group ? group : 16, kStreamK, 0, pl);
  if (rc) return rc;
  if (ws_bytes) *ws_bytes = pl.ws_bytes;
  if (n_counters) *n_counters = pl.counters;
  return FP4X_OK;
}

int fp4x_plan_describe(int fmt, int64_t m, int64_t n, int64_t k, int64_t batch, int group, int whole, char* buf,
                       size_t len) {
  if (fmt < 0 || fmt > 5 || !buf || len == 0) return fail(FP4X_ERR_INVALID_ARG, "bad argument");
  Plan pl;
  int rc = make_plan(fmt, m, n, k, batch, group ? group : 16, whole ? kWholeTile : kStreamK, 0, pl);
  if (rc) return rc;
  snprintf(buf, len,
           "KPW=%d KP=%d KC=%d NCH=%d CPP=%d RT=%d NS=%d STG=%d BI0=%d NB0=%d BI1=%d SB=%d smem=%d whole=%d "
           "ws=%zu counters=%lld ctas=%lld",
           pl.KPW, pl.KP, pl.KC, pl.NCH, pl.CPP, pl.RT, pl.NS, pl.STG, pl.BI0, pl.NB0, pl.BI1, pl.SB, pl.smem_total,
           pl.whole, pl.ws_bytes, (long long)pl.counters, (long long)pl.CPP * pl.KP * batch);
  return FP4X_OK;
}

int fp4x_mx8_linear(const void* x, int64_t x_stride, const void* w, const void* s, void* out, int64_t out_stride,
                    int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                    int64_t n_counters, void* stream) {
  const int rc = run_mx8_tc(x, x_stride, w, s, out, out_stride, out_dtype, m, n, k, stream);
  if (rc <= 0) return rc;
  return run_gemv(FMT_MX8, x, x_stride, w, nullptr, s, 1.f, 16, out, nullptr, out_stride, out_dtype, m, n, k, ws,
                  ws_bytes, counters, n_counters, stream, EPI_STORE);
}

int fp4x_bf16_linear(const void* x, int64_t x_stride, const void* w, void* out, int64_t out_stride, int out_dtype,
                     int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                     int64_t n_counters, void* stream) {
  return run_gemv(FMT_BF16, x, x_stride, w, nullptr, nullptr, 1.f, 16, out, nullptr, out_stride, out_dtype, m, n, k,
                  ws, ws_bytes, counters, n_counters, stream, EPI_STORE);
}

int fp4x_nv4_linear(const void* x, int64_t x_stride, const void* wp, const void* s, float gs, void* out,
                    int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes,
                    int32_t* counters, int64_t n_counters, void* stream) {
  const int rc = run_nv4_tc(x, x_stride, wp, s, gs, out, out_stride, out_dtype, m, n, k, stream);
  if (rc <= 0) return rc;
  return run_gemv(FMT_NV4, x, x_stride, wp, nullptr, s, gs, 16, out, nullptr, out_stride, out_dtype, m, n, k, ws,
                  ws_bytes, counters, n_counters, stream, EPI_STORE);
}

int fp4x_w8_linear(const void* x, int64_t x_stride, const void* q, const void* s, void* out, int64_t out_stride,
                   int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                   int64_t n_counters, void* stream) {
  return run_gemv(FMT_W8, x, x_stride, q, nullptr, s, 1.f, 16, out, nullptr, out_stride, out_dtype, m, n, k, ws,
                  ws_bytes, counters, n_counters, stream, EPI_STORE);
}

int fp4x_w6_linear(const void* x, int64_t x_stride, const void* lo, const void* hi, const void* s, void* out,
                   int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes,
                   int32_t* counters, int64_t n_counters, void* stream) {
  return run_gemv(FMT_W6, x, x_stride, lo, hi, s, 1.f, 16, out, nullptr, out_stride, out_dtype, m, n, k, ws,
                  ws_bytes, counters, n_counters, stream, EPI_STORE);
}

int fp4x_int2_logits(const void* x, int64_t x_stride, const void* p, const void* s, int group, void* out,
                     int64_t out_stride, int out_dtype, void* out_bf16, int64_t m, int64_t n, int64_t k, void* ws,
                     size_t ws_bytes, int32_t* counters, int64_t n_counters, void* stream) {
  const int rc = run_int2_tc(x, x_stride, p, s, group, out, out_bf16, out_stride, out_dtype, m, n, k, stream);
  if (rc <= 0) return rc;
  return run_gemv(FMT_INT2, x, x_stride, p, nullptr, s, 1.f, group, out, out_bf16, out_stride, out_dtype, m, n, k,
                  ws, ws_bytes, counters, n_counters, stream, EPI_HEAD);
}

size_t fp4x_w8_batch_table_bytes(int64_t count) { return (size_t)(count > 0 ? count : 0) * sizeof(BatchEntry); }

int fp4x_w8_batch_prepare(const fp4x_w8_item* items, int64_t count, int64_t n, int64_t k, void* table,
                          size_t table_bytes) {
  if (!items || count < 1 || count > 65535 || !table) return fail(FP4X_ERR_INVALID_ARG, "bad item array");
  if (table_bytes < fp4x_w8_batch_table_bytes(count) || !aligned(table, 64))
    return fail(FP4X_ERR_WORKSPACE, "table too small or not 64-byte aligned (see fp4x_w8_batch_table_bytes)");
  if (k % 64 || n < 1) return fail(FP4X_ERR_UNSUPPORTED, "K must be a multiple of 64");
  Plan pl;
  int rc = make_plan(FMT_W8, 1, n, k, count, 16, kStreamK, 0, pl);
  if (rc) return rc;
  std::vector<BatchEntry> host((size_t)count);
  std::memset(host.data(), 0, host.size() * sizeof(BatchEntry));
  for (int64_t i = 0; i < count; ++i) {
    const fp4x_w8_item& it = items[i];
    if ((rc = check_rows(it.q, k, "weight"))) return rc;
    if (!it.x || !it.s || !it.out || !aligned(it.x, 16) || !aligned(it.s, 4))
      return fail(FP4X_ERR_INVALID_ARG, "bad item pointers");
    if ((rc = encode_rows_uncached(&host[i].tm0, it.q, n, k, pl.BI0))) return rc;
    host[i].x = it.x;
    host[i].sc = (const uint8_t*)it.s;
    host[i].out = it.out;
  }
  cudaError_t e = cudaMemcpy(table, host.data(), host.size() * sizeof(BatchEntry), cudaMemcpyHostToDevice);
  return check_launch(e, "copying the batch table");
}

int fp4x_w8_linear_batched(const void* table, int64_t count, int64_t x_stride, int64_t out_stride, int out_dtype,
                           int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                           int64_t n_counters, void* stream) {
  int rc;
  if (!table || count < 1 || count > 65535) return fail(FP4X_ERR_INVALID_ARG, "bad batch table");
  if ((rc = check_out_dtype(out_dtype))) return rc;
  if (x_stride % 8 || x_stride < k) return fail(FP4X_ERR_UNSUPPORTED, "activation stride must be a multiple of 8 elements");
  Plan pl;
  if ((rc = make_plan(FMT_W8, m, n, k, count, 16, kStreamK, 0, pl))) return rc;
  if ((rc = check_scratch(pl, ws, ws_bytes, counters, n_counters))) return rc;
  Plan p1;
  if ((rc = make_plan(FMT_W8, 1, n, k, count, 16, kStreamK, 0, p1))) return rc;
  if (p1.BI0 != pl.BI0) return fail(FP4X_ERR_UNSUPPORTED, "batch table prepared for a different box width");
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  a.batch = reinterpret_cast<const BatchEntry*>(table);
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = x_stride; a.lds = k / 16; a.scw = 4;  // item scale pointers are only required to be 4-byte aligned
  a.out_stride = out_stride; a.out_dtype = out_dtype; a.post = 1.f; a.group = 16;
  a.ws = (float*)ws; a.sem = counters;
  fill_args(pl, a);
  return launch_nt<FMT_W8, EPI_STORE>(pl, a, count, (cudaStream_t)stream);
}

int fp4x_hc_down(const void* x, int64_t x_stride, const void* q, const void* s, void* di, void* bot, int64_t m,
                 int64_t n, int64_t k, int64_t lr, int64_t hc, void* ws, size_t ws_bytes, int32_t* counters,
                 int64_t n_counters, void* stream) {
  if (!di || !bot) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (lr < 1 || lr > n || hc < 1 || hc > 8) return fail(FP4X_ERR_INVALID_ARG, "bad lr/hc");
  return run_gemv(FMT_W8, x, x_stride, q, nullptr, s, 1.f, 16, di, bot, n, FP4X_BF16, m, n, k, ws, ws_bytes, counters,
                  n_counters, stream, EPI_HC_DOWN, kStreamK, (int)lr, (int)hc);
}

int fp4x_hc_up(const void* bot, int64_t bot_stride, const void* qi, const void* si, const void* nrm,
               int64_t nrm_stride, void* out, int64_t m, int64_t n, int64_t k, int64_t hc, int64_t bj, void* stream) {
  int rc;
  if (!out || !nrm || !si) return fail(FP4X_ERR_INVALID_ARG, "null pointer");
  if (hc < 1 || hc > 8 || bj < 1 || (hc * bj != 16 && hc * bj != 32) || n % (hc * bj) || n % kRB)
    return fail(FP4X_ERR_UNSUPPORTED, "hc * bj must be 16 or 32 and the rows a multiple of 64");
  Plan pl;
  if ((rc = make_plan(FMT_W8, m, n, k, 1, 16, kWholeTile, 1, pl))) return rc;
  if ((rc = check_x(bot, bot_stride, k))) return rc;
  if ((rc = check_rows(qi, k, "weight"))) return rc;
  const int scw = scale_width(si, k / 16, pl.SB);
  if (!scw) return fail(FP4X_ERR_UNSUPPORTED, "scale rows must be 4-byte aligned");
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  if ((rc = encode_rows(&a.tm0, qi, n, k, pl.BI0))) return rc;
  a.item = GemvItem{bot, (const uint8_t*)si, out, nullptr};
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = bot_stride; a.lds = k / 16; a.scw = scw;
  a.out_stride = n / hc; a.out_dtype = FP4X_BF16; a.post = 1.f; a.group = 16;
  a.hc = (int)hc; a.bj = (int)bj; a.nrm = nrm; a.nrm_stride = nrm_stride;
  fill_args(pl, a);
  return launch_nt<FMT_W8, EPI_HC_UP>(pl, a, 1, (cudaStream_t)stream);
}

int fp4x_hc_mixer_unfused(const void* x, int64_t x_stride, const void* qd, const void* sd, const void* qu,
                          const void* su, void* di, void* bot, void* g, void* out, int64_t m, int64_t n_down,
                          int64_t k, int64_t lr, int64_t hc, int64_t n_up, void* ws, size_t ws_bytes,
                          int32_t* counters, int64_t n_counters, void* stream) {
  int rc;
  if (!di || !bot || !g || !out) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (lr < 1 || lr > n_down || hc < 1 || hc > 8 || n_up % hc) return fail(FP4X_ERR_INVALID_ARG, "bad lr/hc/n_up");
  cudaStream_t st = (cudaStream_t)stream;
  // 1. down GEMV with the same plan as the fused kernel; its epilogue writes only di (the cast)
  if ((rc = run_gemv(FMT_W8, x, x_stride, qd, nullptr, sd, 1.f, 16, di, nullptr, n_down, FP4X_BF16, m, n_down, k, ws,
                     ws_bytes, counters, n_counters, stream, EPI_HC_DOWN, kStreamK, (int)lr, (int)hc)))
    return rc;
  // 2. scaled SiLU
  if ((rc = check_launch(launch_pdl(hc_scaled_silu_kernel, dim3(64), dim3(256), 0, st, (const __nv_bfloat16*)di,
                                    (__nv_bfloat16*)bot, (int)m, (int)n_down, (int)lr, (int)hc),
                         "scaled silu")))
    return rc;
  // 3. up GEMV on the original rows, whole-block plan (the same per-row arithmetic as the fused up kernel)
  if ((rc = run_gemv(FMT_W8, bot, lr, qu, nullptr, su, 1.f, 16, g, nullptr, n_up, FP4X_BF16, m, n_up, lr, nullptr, 0,
                     nullptr, 0, stream, EPI_STORE, kWholeTile)))
    return rc;
  // 4. gate-mean
  return check_launch(launch_pdl(hc_gate_mean_kernel, dim3(64), dim3(256), 0, st, (const __nv_bfloat16*)g,
                                 (const __nv_bfloat16*)x, x_stride, (__nv_bfloat16*)out, (int)m, (int)(n_up / hc),
                                 (int)hc),
                      "gate mean");
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------------
// MXFP8 GEMV without caller scratch: split-K partials and arrival counters live in file-scope static device
// arrays of the library (one copy per device).  The counters are zero when the module loads and every completed
// call leaves them zero; the partial tiles are written before they are read.
// ------------------------------------------------------------------------------------------------------
namespace fp4x {

constexpr size_t kStaticWsBytes = size_t(8) << 20;  // 8 MiB of split-K partial tiles
constexpr int64_t kStaticCounters = 32768;          // int32 arrival counters (rows up to 524,288)

static __device__ __align__(256) unsigned char g_static_ws[kStaticWsBytes];
static __device__ __align__(256) int32_t g_static_counters[kStaticCounters];

// device addresses of the static scratch on the current device, resolved on the first call per device
static int static_scratch(void** ws, int32_t** counters) {
  static void* ws_of[64] = {};
  static int32_t* cnt_of[64] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(FP4X_ERR_UNSUPPORTED, "device ordinal above 63");
  std::lock_guard<std::mutex> lk(mu);
  if (!ws_of[dev]) {
    void* w = nullptr;
    void* c = nullptr;
    e = cudaGetSymbolAddress(&w, g_static_ws);
    if (e != cudaSuccess)
      return fail(FP4X_ERR_CUDA, std::string("cudaGetSymbolAddress(static workspace): ") + cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&c, g_static_counters);
    if (e != cudaSuccess)
      return fail(FP4X_ERR_CUDA, std::string("cudaGetSymbolAddress(static counters): ") + cudaGetErrorString(e));
    ws_of[dev] = w;
    cnt_of[dev] = (int32_t*)c;
  }
  *ws = ws_of[dev];
  *counters = cnt_of[dev];
  return FP4X_OK;
}

int reset_static_counters(cudaStream_t st) {
  void* ws = nullptr;
  int32_t* cnt = nullptr;
  int rc = static_scratch(&ws, &cnt);
  if (rc) return rc;
  cudaError_t e = cudaMemsetAsync(cnt, 0, sizeof(int32_t) * kStaticCounters, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, std::string("zeroing the static counters: ") + cudaGetErrorString(e));
  return FP4X_OK;
}

}  // namespace fp4x

extern "C" int fp4x_test_set_static_counter(int64_t index, int32_t value, void* stream) {
  if (index < 0 || index >= kStaticCounters) return fail(FP4X_ERR_INVALID_ARG, "counter index out of range");
  void* ws = nullptr;
  int32_t* cnt = nullptr;
  int rc = static_scratch(&ws, &cnt);
  if (rc) return rc;
  cudaError_t e = cudaMemcpyAsync(cnt + index, &value, sizeof(int32_t), cudaMemcpyHostToDevice, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  return check_launch(e, "writing a static counter");
}

extern "C" int fp4x_mx8_linear_noalloc(const void* x, int64_t x_stride, const void* w, const void* s, void* out,
                                       int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k,
                                       void* stream) {
  int rc;
  if ((rc = check_out_dtype(out_dtype))) return rc;
  Plan pl;
  if ((rc = make_plan(FMT_MX8, m, n, k, 1, 16, kStreamK, 0, pl))) return rc;
  if (pl.ws_bytes > kStaticWsBytes || pl.counters > kStaticCounters)
    return fail(FP4X_ERR_WORKSPACE, "fp4x_mx8_linear_noalloc: this shape needs " + std::to_string(pl.ws_bytes) +
                                        " workspace bytes and " + std::to_string(pl.counters) +
                                        " counters; the static scratch holds " + std::to_string(kStaticWsBytes) +
                                        " bytes and " + std::to_string(kStaticCounters) + " counters");
  if ((rc = check_x(x, x_stride, k))) return rc;
  if ((rc = check_rows(w, k, "weight"))) return rc;
  if (!s) return fail(FP4X_ERR_INVALID_ARG, "null scales");
  const int64_t lds = k / 32;
  const int scw = scale_width(s, lds, pl.SB);
  if (!scw) return fail(FP4X_ERR_UNSUPPORTED, "scale rows must be 4-byte aligned");
  if (!out) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (out_stride < n) return fail(FP4X_ERR_INVALID_ARG, "out_stride < n");
  void* ws = nullptr;
  int32_t* counters = nullptr;
  if ((rc = static_scratch(&ws, &counters))) return rc;
  GemvArgs a;
  std::memset(&a, 0, sizeof(a));
  if ((rc = encode_rows_uncached(&a.tm0, w, n, k, pl.BI0))) return rc;
  a.item = GemvItem{x, (const uint8_t*)s, out, nullptr};
  a.batch = nullptr;
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = x_stride; a.lds = lds; a.scw = scw;
  a.out_stride = out_stride; a.out_dtype = out_dtype; a.post = 1.f; a.group = 16;
  a.ws = (float*)ws; a.sem = counters;
  fill_args(pl, a);
  return launch_nt<FMT_MX8, EPI_STORE>(pl, a, 1, (cudaStream_t)stream);
}
