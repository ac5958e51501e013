// Host planner, launchers and C ABI of the GEMV family (MXFP8, W8, W6, NVFP4, BF16, INT2, batched W8 and the
// fused / unfused hyper-connection mixer).
#include <mutex>
#include <string>

#include "fp4x_gemv.cuh"
#include "fp4x_host.h"

namespace fp4x {

__device__ int g_dev_error = 0;

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
    if (f.sms <= 0) f.sms = 148;
    if (f.smem_optin <= 0) f.smem_optin = 227 * 1024;
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
  if (e == cudaSuccess && n < 512) tab[n++] = Entry{kernel, dev, bytes};
  return e;
}

// ------------------------------------------------------------------------------------------------------
// planning
// ------------------------------------------------------------------------------------------------------
enum PlanMode { kStreamK = 0, kWholeTile = 1 };

struct Plan {
  int NT, RG, RU, MP;
  int KPW, KP, KC, NCH, CPP, RT, NS, SMAX, whole;
  int P0, P1, PS, STG, XP;
  int smem_x, smem_stage, smem_scr, smem_total;
  size_t ws_bytes;
  int64_t counters;
};

static int round_up(int v, int a) { return (v + a - 1) / a * a; }
static int pitch_for(int bytes, int mod) {
  if (bytes == 0) return 0;
  int p = round_up(bytes, 16);
  while (p % 128 != mod) p += 16;
  return p;
}

static double bytes_per_k(int fmt, int group) {
  const FmtGeom G = fmt_geom(fmt);
  double b = (double)G.n0 / G.d0 + (G.n1 ? (double)G.n1 / G.d1 : 0.0);
  if (G.sn) b += fmt == FMT_INT2 ? 2.0 / group : (double)G.sn / G.sd;
  return b;
}

// returns 0 and fills `pl`, or a negative status
static int make_plan(int fmt, int64_t M, int64_t N, int64_t K, int64_t batch, int group, PlanMode mode, int RG,
                     int epi_scratch, Plan& pl) {
  if (M < 1 || M > 16) return fail(FP4X_ERR_INVALID_ARG, "M must be in 1..16 (decode shapes)");
  if (N < 1 || K < 1 || batch < 1) return fail(FP4X_ERR_INVALID_ARG, "empty shape");
  if (N > (1 << 30) || K > (1 << 20)) return fail(FP4X_ERR_UNSUPPORTED, "shape too large");
  const FmtGeom G = fmt_geom(fmt);
  if (fmt == FMT_INT2 && group != 16 && group != 32) return fail(FP4X_ERR_UNSUPPORTED, "INT2 group must be 16 or 32");
  if (K % 64 != 0 || K % G.blk != 0)
    return fail(FP4X_ERR_UNSUPPORTED, "K=" + std::to_string(K) + " must be a multiple of 64 and of " + std::to_string(G.blk));
  if (fmt == FMT_MX8 && K % 128 != 0) return fail(FP4X_ERR_UNSUPPORTED, "MXFP8 needs K % 128 == 0");
  const DeviceFacts& dv = device_facts();
  pl.NT = M <= 8 ? 1 : 2;
  pl.MP = 8 * pl.NT;
  pl.RG = RG;
  pl.RU = 16 * RG;
  pl.RT = (int)((N + pl.RU - 1) / pl.RU);
  const int G_ctas = dv.sms;
  // INT2 heads always use whole row tiles: each row's fp32 sum then has a fixed order that does not depend on the
  // vocabulary size or the grid, so a vocab-sharded head reproduces the unsharded coarse values bit for bit
  const bool whole = (mode == kWholeTile || K % 256 != 0 || fmt == FMT_INT2);
  pl.whole = whole ? 1 : 0;
  if (!whole) {
    // panel width: the activation staging per CTA should stay small next to the CTA's share of the weights
    const double share = (double)batch * N * K * bytes_per_k(fmt, group) / G_ctas;
    const double xbudget = share / 4 > 8192 ? share / 4 : 8192;
    int best = 256;
    for (int kpw = 256; kpw <= K; kpw += 256) {
      if (K % kpw) continue;
      if ((double)kpw * pl.MP * 2 <= xbudget && kpw * pl.MP * 2 <= 96 * 1024) best = kpw;
    }
    pl.KPW = best;
    pl.KP = (int)(K / best);
    pl.KC = 256;
    pl.NCH = best / 256;
  } else {
    pl.KP = 1;
    pl.KPW = (int)K;
    pl.KC = 0;  // chosen below with the stage geometry
  }
  const int64_t Up = (int64_t)pl.RT * (whole ? 1 : pl.NCH);
  int64_t cpp = G_ctas / (pl.KP * batch);
  if (cpp < 1) cpp = 1;
  if (!whole && pl.NCH > 1) {
    // row tiles shared between warps need every warp of a panel to own at least one chunk unit
    if (cpp * kWarps > Up) cpp = Up / kWarps > 0 ? Up / kWarps : 1;
    if (cpp * kWarps > Up) return fail(FP4X_ERR_UNSUPPORTED, "too few chunk units for one CTA");
  } else if (cpp > (Up + 1) / 2) {
    cpp = (Up + 1) / 2;  // whole row tiles: about two per CTA at least
  }
  pl.CPP = (int)cpp;
  // stage geometry
  const int sd = fmt == FMT_INT2 ? group / 2 : G.sd;
  pl.XP = (pl.KPW / 16) * 32 + 32;
  pl.smem_x = 640;
  pl.smem_scr = round_up(pl.smem_x + pl.MP * pl.XP, 128);
  const int scr_bytes = epi_scratch ? kWarps * pl.RU * pl.MP * 4 : 0;
  pl.smem_stage = round_up(pl.smem_scr + scr_bytes, 128);
  const int cap = dv.smem_optin;
  auto geom = [&](int kc, int& ns) {
    const int pb0 = kc * G.n0 / G.d0;
    const int pb1 = G.n1 ? kc * G.n1 / G.d1 : 0;
    const int sb = G.sn ? kc * G.sn / sd : 0;
    pl.P0 = pitch_for(pb0, G.mod0);
    pl.P1 = pitch_for(pb1, G.mod1);
    pl.PS = sb;
    pl.STG = round_up(pl.RU * (pl.P0 + pl.P1 + pl.PS), 128);
    ns = (cap - pl.smem_stage) / (kWarps * pl.STG);
    return sb % 4 == 0;
  };
  int ns = 0;
  if (whole) {
    // largest chunk (a multiple of the decode block dividing K) that still leaves a 3-deep ring, else 2-deep
    const int step = G.blk > 64 ? G.blk : 64;
    int pick = 0;
    for (int want = 3; want >= 2 && !pick; --want)
      for (int kc = (int)K; kc >= step; kc -= step) {
        if (K % kc || kc % step) continue;
        int n2;
        if (geom(kc, n2) && n2 >= want) { pick = kc; break; }
      }
    if (!pick) return fail(FP4X_ERR_UNSUPPORTED, "shape needs more shared memory than available");
    pl.KC = pick;
    pl.NCH = (int)(K / pick);
  }
  if (!geom(pl.KC, ns)) return fail(FP4X_ERR_UNSUPPORTED, "scale row chunk must be a multiple of 4 bytes");
  if (ns > kMaxStages) ns = kMaxStages;
  if (ns < 2) return fail(FP4X_ERR_UNSUPPORTED, "shape needs more shared memory than available (K too large?)");
  pl.NS = ns;
  pl.smem_total = pl.smem_stage + kWarps * ns * pl.STG;
  const int Wp = pl.CPP * kWarps;
  pl.SMAX = whole ? 1 : (int)((int64_t)(pl.NCH - 1) * Wp / Up) + 2;
  if (pl.SMAX > Wp) pl.SMAX = Wp;
  const size_t slot = (size_t)pl.RU * pl.MP * sizeof(float);
  if (pl.KP > 1)
    pl.ws_bytes = (size_t)batch * pl.KP * pl.RT * pl.SMAX * slot;
  else if (pl.NCH > 1 && !whole)
    pl.ws_bytes = (size_t)batch * Wp * 2 * slot;
  else
    pl.ws_bytes = 0;
  pl.counters = (pl.KP > 1 || (pl.NCH > 1 && !whole)) ? (int64_t)batch * pl.RT : 0;
  return FP4X_OK;
}

// ------------------------------------------------------------------------------------------------------
// launch
// ------------------------------------------------------------------------------------------------------
template <int FMT, int NT, int RG, int EPI>
static int launch_t(const Plan& pl, GemvArgs& a, int64_t batch, cudaStream_t st) {
  auto kern = gemv_kernel<FMT, NT, RG, EPI>;
  cudaError_t e = ensure_smem_attr((const void*)kern, pl.smem_total);
  if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute");
  return check_launch(launch_pdl(kern, dim3(pl.CPP, pl.KP, (unsigned)batch), dim3(kThreads), pl.smem_total, st, a),
                      "gemv launch");
}

template <int FMT, int EPI, int RG>
static int launch_nt(const Plan& pl, GemvArgs& a, int64_t batch, cudaStream_t st) {
  return pl.NT == 1 ? launch_t<FMT, 1, RG, EPI>(pl, a, batch, st) : launch_t<FMT, 2, RG, EPI>(pl, a, batch, st);
}

static void fill_args(const Plan& pl, GemvArgs& a) {
  a.err = dev_error_ptr();
  a.KPW = pl.KPW; a.KP = pl.KP; a.KC = pl.KC; a.NCH = pl.NCH; a.CPP = pl.CPP; a.RT = pl.RT; a.NS = pl.NS;
  a.SMAX = pl.SMAX; a.whole = pl.whole; a.P0 = pl.P0; a.P1 = pl.P1; a.PS = pl.PS; a.STG = pl.STG; a.XP = pl.XP;
  a.smem_x = pl.smem_x; a.smem_stage = pl.smem_stage; a.smem_scr = pl.smem_scr;
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
                    void* stream, int epi, PlanMode mode = kStreamK) {
  int rc;
  if ((rc = check_out_dtype(out_dtype))) return rc;
  Plan pl;
  if ((rc = make_plan(fmt, m, n, k, 1, group, mode, 1, 0, pl))) return rc;
  if ((rc = check_x(x, x_stride, k))) return rc;
  const FmtGeom G = fmt_geom(fmt);
  const int64_t ld0 = k * G.n0 / G.d0, ld1 = G.n1 ? k * G.n1 / G.d1 : 0;
  const int sd = fmt == FMT_INT2 ? group / 2 : G.sd;
  const int64_t lds = G.sn ? k * G.sn / sd : 0;
  if ((rc = check_rows(p0, ld0, "weight"))) return rc;
  if (G.n1 && (rc = check_rows(p1, ld1, "weight plane 1"))) return rc;
  if (G.sn && (!sc || !aligned(sc, 4) || lds % 4)) return fail(FP4X_ERR_UNSUPPORTED, "scales must be 4-byte aligned rows");
  if (!out) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (out_stride < n) return fail(FP4X_ERR_INVALID_ARG, "out_stride < n");
  if ((rc = check_scratch(pl, ws, ws_bytes, counters, n_counters))) return rc;
  GemvArgs a = {};
  a.item = GemvItem{x, (const uint8_t*)p0, (const uint8_t*)p1, (const uint8_t*)sc, out, out2};
  a.items4 = nullptr;
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = x_stride; a.ld0 = ld0; a.ld1 = ld1; a.lds = lds;
  a.out_stride = out_stride; a.out_dtype = out_dtype; a.post = post; a.group = group;
  a.ws = (float*)ws; a.sem = counters;
  fill_args(pl, a);
  cudaStream_t st = (cudaStream_t)stream;
  switch (fmt) {
    case FMT_MX8: return launch_nt<FMT_MX8, EPI_STORE, 1>(pl, a, 1, st);
    case FMT_W8:
      if (epi == EPI_HC_DOWN) return launch_nt<FMT_W8, EPI_HC_DOWN, 1>(pl, a, 1, st);
      return launch_nt<FMT_W8, EPI_STORE, 1>(pl, a, 1, st);
    case FMT_W6: return launch_nt<FMT_W6, EPI_STORE, 1>(pl, a, 1, st);
    case FMT_NV4: return launch_nt<FMT_NV4, EPI_STORE, 1>(pl, a, 1, st);
    case FMT_BF16: return launch_nt<FMT_BF16, EPI_STORE, 1>(pl, a, 1, st);
    case FMT_INT2: return launch_nt<FMT_INT2, EPI_HEAD, 1>(pl, a, 1, st);
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

}  // namespace fp4x

using namespace fp4x;

// ------------------------------------------------------------------------------------------------------
// C ABI
// ------------------------------------------------------------------------------------------------------
extern "C" {

int fp4x_version(void) { return 100; }

const char* fp4x_last_error_message(void) { return t_msg.c_str(); }

int fp4x_device_error(void* stream, int clear, int* code_out) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_dev_error, sizeof(int), 0, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, std::string("reading the device error word: ") + cudaGetErrorString(e));
  if (code_out) *code_out = v;
  if (clear && v) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_dev_error, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize((cudaStream_t)stream);
    if (e != cudaSuccess) return fail(FP4X_ERR_CUDA, cudaGetErrorString(e));
  }
  return v ? fail(FP4X_ERR_DEVICE, "device error word = " + std::to_string(v)) : FP4X_OK;
}

int fp4x_gemv_query(int fmt, int64_t m, int64_t n, int64_t k, int64_t batch, int group, size_t* ws_bytes,
                    int64_t* n_counters) {
  if (fmt < 0 || fmt > 5) return fail(FP4X_ERR_INVALID_ARG, "bad format");
  Plan pl;
  int rc = make_plan(fmt, m, n, k, batch, group ? group : 16, kStreamK, 1, 0, pl);
  if (rc) return rc;
  if (ws_bytes) *ws_bytes = pl.ws_bytes;
  if (n_counters) *n_counters = pl.counters;
  return FP4X_OK;
}

int fp4x_mx8_linear(const void* x, int64_t x_stride, const void* w, const void* s, void* out, int64_t out_stride,
                    int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes, int32_t* counters,
                    int64_t n_counters, void* stream) {
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
  return run_gemv(FMT_INT2, x, x_stride, p, nullptr, s, 1.f, group, out, out_bf16, out_stride, out_dtype, m, n, k,
                  ws, ws_bytes, counters, n_counters, stream, EPI_HEAD);
}

int fp4x_w8_linear_batched(const fp4x_w8_item* items, int64_t count, int64_t x_stride, int64_t out_stride,
                           int out_dtype, int64_t m, int64_t n, int64_t k, void* ws, size_t ws_bytes,
                           int32_t* counters, int64_t n_counters, void* stream) {
  int rc;
  if (!items || count < 1 || count > 65535) return fail(FP4X_ERR_INVALID_ARG, "bad item array");
  if ((rc = check_out_dtype(out_dtype))) return rc;
  if (x_stride % 8 || x_stride < k || k % 16) return fail(FP4X_ERR_UNSUPPORTED, "activation stride must be a multiple of 8 elements");
  Plan pl;
  if ((rc = make_plan(FMT_W8, m, n, k, count, 16, kStreamK, 1, 0, pl))) return rc;
  if ((rc = check_scratch(pl, ws, ws_bytes, counters, n_counters))) return rc;
  static_assert(sizeof(fp4x_w8_item) == 4 * sizeof(void*), "item layout is four pointers {x, q, s, out}");
  GemvArgs a = {};
  a.items4 = reinterpret_cast<const void* const*>(items);
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = x_stride; a.ld0 = k; a.ld1 = 0; a.lds = k / 16;
  a.out_stride = out_stride; a.out_dtype = out_dtype; a.post = 1.f; a.group = 16;
  a.ws = (float*)ws; a.sem = counters;
  fill_args(pl, a);
  return launch_nt<FMT_W8, EPI_STORE, 1>(pl, a, count, (cudaStream_t)stream);
}

int fp4x_hc_down(const void* x, int64_t x_stride, const void* q, const void* s, void* di, void* bot, int64_t m,
                 int64_t n, int64_t k, int64_t lr, int64_t hc, void* ws, size_t ws_bytes, int32_t* counters,
                 int64_t n_counters, void* stream) {
  if (!di || !bot) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (lr < 1 || lr > n || hc < 1 || hc > 8) return fail(FP4X_ERR_INVALID_ARG, "bad lr/hc");
  int rc;
  Plan pl;
  if ((rc = make_plan(FMT_W8, m, n, k, 1, 16, kStreamK, 1, 0, pl))) return rc;
  if ((rc = check_x(x, x_stride, k))) return rc;
  if ((rc = check_rows(q, k, "weight"))) return rc;
  if ((rc = check_scratch(pl, ws, ws_bytes, counters, n_counters))) return rc;
  GemvArgs a = {};
  a.item = GemvItem{x, (const uint8_t*)q, nullptr, (const uint8_t*)s, di, bot};
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = x_stride; a.ld0 = k; a.lds = k / 16;
  a.out_stride = n; a.out_dtype = FP4X_BF16; a.post = 1.f; a.group = 16;
  a.lr = (int)lr; a.hc = (int)hc;
  a.ws = (float*)ws; a.sem = counters;
  fill_args(pl, a);
  return launch_nt<FMT_W8, EPI_HC_DOWN, 1>(pl, a, 1, (cudaStream_t)stream);
}

static int hc_up_impl(const void* bot, int64_t bot_stride, const void* qi, const void* si, const void* nrm,
                      int64_t nrm_stride, void* out, int64_t m, int64_t n, int64_t k, int64_t hc, int64_t bj,
                      void* stream) {
  int rc;
  if (!out || !nrm) return fail(FP4X_ERR_INVALID_ARG, "null pointer");
  if (hc < 1 || hc > 8 || bj < 1 || (hc * bj != 16 && hc * bj != 32) || n % (hc * bj))
    return fail(FP4X_ERR_UNSUPPORTED, "hc * bj must be 16 or 32 and divide n");
  const int RG = (int)(hc * bj / 16);
  Plan pl;
  if ((rc = make_plan(FMT_W8, m, n, k, 1, 16, kWholeTile, RG, 1, pl))) return rc;
  if ((rc = check_x(bot, bot_stride, k))) return rc;
  if ((rc = check_rows(qi, k, "weight"))) return rc;
  GemvArgs a = {};
  a.item = GemvItem{bot, (const uint8_t*)qi, nullptr, (const uint8_t*)si, out, nullptr};
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.x_stride = bot_stride; a.ld0 = k; a.lds = k / 16;
  a.out_stride = n / hc; a.out_dtype = FP4X_BF16; a.post = 1.f; a.group = 16;
  a.hc = (int)hc; a.bj = (int)bj; a.nrm = nrm; a.nrm_stride = nrm_stride;
  fill_args(pl, a);
  cudaStream_t st = (cudaStream_t)stream;
  return RG == 1 ? launch_nt<FMT_W8, EPI_HC_UP, 1>(pl, a, 1, st) : launch_nt<FMT_W8, EPI_HC_UP, 2>(pl, a, 1, st);
}

int fp4x_hc_up(const void* bot, int64_t bot_stride, const void* qi, const void* si, const void* nrm,
               int64_t nrm_stride, void* out, int64_t m, int64_t n, int64_t k, int64_t hc, int64_t bj, void* stream) {
  return hc_up_impl(bot, bot_stride, qi, si, nrm, nrm_stride, out, m, n, k, hc, bj, stream);
}

int fp4x_hc_mixer_unfused(const void* x, int64_t x_stride, const void* qd, const void* sd, const void* qu,
                          const void* su, void* di, void* bot, void* g, void* out, int64_t m, int64_t n_down,
                          int64_t k, int64_t lr, int64_t hc, int64_t n_up, void* ws, size_t ws_bytes,
                          int32_t* counters, int64_t n_counters, void* stream) {
  int rc;
  if (!di || !bot || !g || !out) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (lr < 1 || lr > n_down || hc < 1 || hc > 8 || n_up % hc) return fail(FP4X_ERR_INVALID_ARG, "bad lr/hc/n_up");
  cudaStream_t st = (cudaStream_t)stream;
  // 1. down GEMV with the same plan as the fused kernel; epilogue writes only di (the cast)
  if ((rc = run_gemv(FMT_W8, x, x_stride, qd, nullptr, sd, 1.f, 16, di, nullptr, n_down, FP4X_BF16, m, n_down, k,
                     ws, ws_bytes, counters, n_counters, stream, EPI_HC_DOWN)))
    return rc;
  // (run_gemv's HC_DOWN epilogue takes lr/hc from the args; with bot == nullptr only di is stored)
  // 2. scaled SiLU
  if ((rc = check_launch(launch_pdl(hc_scaled_silu_kernel, dim3(64), dim3(256), 0, st, (const __nv_bfloat16*)di,
                                    (__nv_bfloat16*)bot, (int)m, (int)n_down, (int)lr, (int)hc),
                         "scaled silu")))
    return rc;
  // 3. up GEMV on the original rows, whole-tile plan (same per-row arithmetic as the fused up kernel)
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
