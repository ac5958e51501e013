// Launchers of the tcgen05 GEMVs (block-scaled NVFP4 / MXFP8 and the INT2 head pass): shape gates, shared-memory
// layout and kernel selection by token count.
#include <algorithm>
#include <cstring>

#include "fp4x_launch.cuh"
#include "fp4x_tc.cuh"
#include "fp4x_tc_int2.cuh"

namespace fp4x {

static int round_up(int v, int a) { return (v + a - 1) / a * a; }

static int check_out_dtype(int d) {
  if (d != FP4X_BF16 && d != FP4X_F16 && d != FP4X_F32) return fail(FP4X_ERR_INVALID_ARG, "bad out_dtype");
  return FP4X_OK;
}

template <int MT>
static int launch_nv4_tc(const tc::Args& a, unsigned grid, int smem_total, void* stream) {
  auto kern = tc::nv4_tc_kernel<MT>;
  cudaError_t e = ensure_smem_attr((const void*)kern, smem_total);
  if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute");
  return check_launch(
      launch_pdl(kern, dim3(grid), dim3(tc::nv_threads(MT)), (size_t)smem_total, (cudaStream_t)stream, a),
      "nv4 tcgen05 launch");
}

// NVFP4 on tcgen05 block-scaled MMAs (fp4x_tc.cuh): M <= 16 tokens (9-16 run the 12- or 16-token kernel), at least
// 64 row blocks of 128, K a multiple of 256.  Returns 1 when the shape is not covered (the caller then uses the
// register-decode kernel).
int run_nv4_tc(const void* x, int64_t x_stride, const void* wp, const void* sc, float gs, void* out,
                      int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* stream) {
  const DeviceFacts& dv = device_facts();
  if (m < 1 || m > tc::kMaxM || k % tc::kKC != 0 || k / tc::kKC > tc::kMaxSlabs || n < 64 * tc::kRows ||
      n > (1 << 30))
    return 1;
  const int mt = m <= 8 ? (int)m : (m <= 12 ? 12 : 16);  // the kernel's token count
  const int NB = (tc::kTerms * mt + 15) / 16 * 16;
  if (4 * (k / 64) > tc::kTmemCols - tc::kColSFB || NB > tc::kColSFA) return 1;
  if (!aligned(x, 16) || x_stride % 8 != 0 || x_stride < k || !aligned(wp, 16) || (k / 2) % 16 != 0) return 1;
  const int64_t lds = k / 16;
  if (lds % 16 != 0 || !aligned(sc, 16) || !out || out_stride < n) return 1;
  int rc;
  if ((rc = check_out_dtype(out_dtype))) return rc;
  tc::Args a;
  std::memset(&a, 0, sizeof(a));
  const int b_bytes = (int)(k / 256) * NB * 128;
  const int xraw = mt > 8 ? 0 : round_up((int)(m * k * 2), 1024);  // more than 8 tokens are read through L2
  const int sfb = round_up((int)(k / 64) * 512, 1024);  // B scales in tcgen05.cp groups, one per 64-k block
  const int fixed = b_bytes + xraw + sfb + tc::kMiscBytes + 1024;
  int ns = (dv.smem_optin - fixed) / tc::kStageBytes;
  if (ns > tc::kMaxStages) ns = tc::kMaxStages;
  if (ns > (int)(k / tc::kKC)) ns = (int)(k / tc::kKC);
  // six stages (96 KB of weights in flight) keep the standalone time (8.16 µs at 16384 x 2560, M = 3) and leave
  // shared memory to the next launch in a decode chain: the C5 step took 2.388 against 2.398 ms with eight
  if (ns > 6) ns = 6;
  if (ns < 2) return 1;
  a.NS = ns;
  a.smem_b = ns * tc::kStageBytes;          // multiple of 1024
  a.smem_xraw = a.smem_b + b_bytes;
  a.smem_sfb = a.smem_xraw + xraw;
  a.smem_misc = a.smem_sfb + sfb;
  const int smem_total = a.smem_misc + tc::kMiscBytes + 1024;
  if ((rc = encode_rows(&a.tm, wp, n, k / 2, 128))) return rc;
  if ((rc = encode_scale_box(&a.tms, sc, n, k / 16, 16))) return rc;
  a.x = (const __nv_bfloat16*)x; a.x_stride = x_stride;
  a.sc = (const uint8_t*)sc; a.lds = lds; a.scw = 16;
  a.out = out; a.out_stride = out_stride; a.out_dtype = out_dtype; a.gs = gs;
  a.M = (int)m; a.N = (int)n; a.K = (int)k; a.NB = NB;
  a.err = dev_error_ptr();
  a.tl = timeline_next();
  const unsigned grid = (unsigned)((n + tc::kRows - 1) / tc::kRows);
  switch (m) {
    case 1: return launch_nv4_tc<1>(a, grid, smem_total, stream);
    case 2: return launch_nv4_tc<2>(a, grid, smem_total, stream);
    case 3: return launch_nv4_tc<3>(a, grid, smem_total, stream);
    case 4: return launch_nv4_tc<4>(a, grid, smem_total, stream);
    case 5: return launch_nv4_tc<5>(a, grid, smem_total, stream);
    case 6: return launch_nv4_tc<6>(a, grid, smem_total, stream);
    case 7: return launch_nv4_tc<7>(a, grid, smem_total, stream);
    case 8: return launch_nv4_tc<8>(a, grid, smem_total, stream);
    default: return mt == 12 ? launch_nv4_tc<12>(a, grid, smem_total, stream)
                             : launch_nv4_tc<16>(a, grid, smem_total, stream);
  }
}

template <int MT>
static int launch_mx8_tc(const tc::MxArgs& a, unsigned grid, int smem_total, void* stream) {
  auto kern = tc::mx8_tc_kernel<MT>;
  cudaError_t e = ensure_smem_attr((const void*)kern, smem_total);
  if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute");
  return check_launch(
      launch_pdl(kern, dim3(grid), dim3(tc::mx_threads(MT)), (size_t)smem_total, (cudaStream_t)stream, a),
      "mx8 tcgen05 launch");
}

// MXFP8 on tcgen05 block-scaled MMAs (fp4x_tc.cuh): M <= 16 tokens (9-16 run the 12- or 16-token kernel), at least
// 64 row blocks of 128, K a multiple of 512 up to 4096.  Returns 1 when the shape is not covered (the caller then uses
// the register-decode kernel).
int run_mx8_tc(const void* x, int64_t x_stride, const void* w, const void* sc, void* out, int64_t out_stride,
                      int out_dtype, int64_t m, int64_t n, int64_t k, void* stream) {
  const DeviceFacts& dv = device_facts();
  if (m < 1 || m > tc::kMxMaxM || k % 512 != 0 || k / tc::kMxKC > tc::kMxMaxChunks || n < 64 * tc::kRows ||
      n > (1 << 30))
    return 1;
  if (!aligned(x, 16) || x_stride % 8 != 0 || x_stride < k || !aligned(w, 16) || !aligned(sc, 16) || !out ||
      out_stride < n)
    return 1;
  int rc;
  if ((rc = check_out_dtype(out_dtype))) return rc;
  const int mt = m <= 8 ? (int)m : (m <= 12 ? 12 : 16);  // the kernel's token count
  const int NB = (tc::kMxTerms * mt + 15) / 16 * 16;
  tc::MxArgs a;
  std::memset(&a, 0, sizeof(a));
  const int b_bytes = (int)(k / tc::kMxKC) * NB * 128;
  const int xraw = mt > 8 ? 0 : round_up((int)(m * k * 2), 1024);  // more than 8 tokens are read through L2
  const int sfb = round_up((int)(k / tc::kMxKC) * 512, 1024);
  const int sfa = round_up(tc::kRows * (int)(k / 32), 1024);
  const int misc = 1024;
  const int fixed = b_bytes + xraw + sfb + sfa + misc + 1024;
  int ns = (dv.smem_optin - fixed) / tc::kStageA;
  if (ns > tc::kMxMaxStages) ns = tc::kMxMaxStages;
  if (ns > (int)(k / tc::kMxKC)) ns = (int)(k / tc::kMxKC);
  if (ns < 2) return 1;
  a.NS = ns;
  a.smem_b = ns * tc::kStageA;
  a.smem_xraw = a.smem_b + b_bytes;
  a.smem_sfb = a.smem_xraw + xraw;
  a.smem_sfa = a.smem_sfb + sfb;
  a.smem_misc = a.smem_sfa + sfa;
  const int smem_total = a.smem_misc + misc + 1024;
  if ((rc = encode_rows(&a.tm, w, n, k, 128))) return rc;
  if ((rc = encode_scale_box(&a.tms, sc, n, k / 32, (int)(k / 32)))) return rc;
  a.x = (const __nv_bfloat16*)x; a.x_stride = x_stride;
  a.out = out; a.out_stride = out_stride; a.out_dtype = out_dtype;
  a.M = (int)m; a.N = (int)n; a.K = (int)k;
  a.err = dev_error_ptr();
  a.tl = timeline_next();
  const unsigned grid = (unsigned)((n + tc::kRows - 1) / tc::kRows);
  switch (m) {
    case 1: return launch_mx8_tc<1>(a, grid, smem_total, stream);
    case 2: return launch_mx8_tc<2>(a, grid, smem_total, stream);
    case 3: return launch_mx8_tc<3>(a, grid, smem_total, stream);
    case 4: return launch_mx8_tc<4>(a, grid, smem_total, stream);
    case 5: return launch_mx8_tc<5>(a, grid, smem_total, stream);
    case 6: return launch_mx8_tc<6>(a, grid, smem_total, stream);
    case 7: return launch_mx8_tc<7>(a, grid, smem_total, stream);
    case 8: return launch_mx8_tc<8>(a, grid, smem_total, stream);
    default: return mt == 12 ? launch_mx8_tc<12>(a, grid, smem_total, stream)
                             : launch_mx8_tc<16>(a, grid, smem_total, stream);
  }
}

// INT2 head logits on tcgen05 (fp4x_tc_int2.cuh): M <= 16 tokens, at least 32 row tiles of 128, groups of 16 or
// 32, K a multiple of 256 with the B operand (K x 32 bytes) fitting beside the stages.  Returns 1 when the shape is
// not covered (the caller then uses the register-decode kernel).
int run_int2_tc(const void* x, int64_t x_stride, const void* p, const void* s, int group, void* out,
                       void* out_bf16, int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k,
                       void* stream) {
  const DeviceFacts& dv = device_facts();
  if (m < 1 || m > tc::kI2MaxM || (group != 16 && group != 32) || k % tc::kI2KC != 0 || n < 32 * tc::kRows ||
      n > (1 << 30))
    return 1;
  if (!aligned(x, 16) || x_stride % 8 != 0 || x_stride < k || !aligned(p, 16) || !aligned(s, 16) || !out ||
      out_stride < n)
    return 1;
  int rc;
  if ((rc = check_out_dtype(out_dtype))) return rc;
  const int b_bytes = (int)(k / 64) * 2048;
  const int misc = 1024;
  const int fixed = b_bytes + misc + 1024;
  int ns = (dv.smem_optin - fixed) / tc::kI2StageBytes;
  if (ns > tc::kI2MaxStages) ns = tc::kI2MaxStages;
  if (ns < 4) return 1;
  tc::I2Args a;
  std::memset(&a, 0, sizeof(a));
  a.NS = ns;
  a.smem_b = ns * tc::kI2StageBytes;  // multiple of 1024
  a.smem_misc = a.smem_b + b_bytes;
  const int smem_total = a.smem_misc + misc + 1024;
  if ((rc = encode_box(&a.tm, p, n, k / 4, 64, tc::kRows))) return rc;
  if ((rc = encode_box(&a.tms, s, n, 2 * k / group, 512 / group, tc::kRows))) return rc;
  a.x = (const __nv_bfloat16*)x; a.x_stride = x_stride;
  a.out = out; a.out_bf16 = out_bf16; a.out_stride = out_stride; a.out_dtype = out_dtype;
  a.M = (int)m; a.N = (int)n; a.K = (int)k; a.group = group;
  a.tiles = (int)((n + tc::kRows - 1) / tc::kRows);
  a.err = dev_error_ptr();
  a.tl = timeline_next();
  const unsigned grid = (unsigned)std::min(a.tiles, dv.sms);
  auto kern = tc::int2_tc_kernel;
  cudaError_t e = ensure_smem_attr((const void*)kern, smem_total);
  if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute");
  return check_launch(launch_pdl(kern, dim3(grid), dim3(tc::kI2Threads), (size_t)smem_total, (cudaStream_t)stream, a),
                      "int2 tcgen05 launch");
}

}  // namespace fp4x
