// Launch plan of the GEMV template and its launchers.  The launchers are templates over (format, epilogue); each
// instantiation lives in its own translation unit (fp4x_inst_*.cu) so the large kernel bodies compile in parallel.
#pragma once
#include "fp4x_gemv.cuh"
#include "fp4x_host.h"

namespace fp4x {

struct Plan {
  int NT, MP;
  int KPW, KP, KC, NCH, CPP, RT, NS, SMAX, whole;
  int BI0, BI1, NB0, SB, STG, off_p1, off_sc, XP;
  int smem_x, smem_misc, smem_scr, smem_xraw, smem_comb, smem_red, smem_total;
  int xdirect;  // 16-token plans: the raw activation panel stays in global memory
  int cluster;
  size_t ws_bytes;
  int64_t counters;
};

// TMA descriptors of [rows][row_bytes] u8 matrices (fp4x_gemv.cu): swizzled 64-row boxes of `inner` bytes (cached per
// pointer and shape), unswizzled 128-row scale boxes, and boxes of any height (64-byte swizzle for 64-byte boxes)
int encode_rows(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int inner);
int encode_scale_box(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int box_bytes);
int encode_box(CUtensorMap* tm, const void* ptr, int64_t rows, int64_t row_bytes, int box_bytes, int box_rows);

// tcgen05 GEMVs (fp4x_tc.cu): 0 or a negative status when launched, 1 when the shape is not covered (the caller
// then runs the register-decode GEMV)
int run_nv4_tc(const void* x, int64_t x_stride, const void* wp, const void* sc, float gs, void* out,
               int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* stream);
int run_mx8_tc(const void* x, int64_t x_stride, const void* w, const void* sc, void* out, int64_t out_stride,
               int out_dtype, int64_t m, int64_t n, int64_t k, void* stream);
int run_int2_tc(const void* x, int64_t x_stride, const void* p, const void* s, int group, void* out, void* out_bf16,
                int64_t out_stride, int out_dtype, int64_t m, int64_t n, int64_t k, void* stream);

// allow clusters of up to 16 CTAs for a kernel, once per (kernel, device)
cudaError_t ensure_nonportable_cluster(const void* kernel);

template <int FMT, int NT, int EPI, int SHAPE>
int launch_s(const Plan& pl, const GemvArgs& a, int64_t batch, cudaStream_t st) {
  const bool wide = (int64_t)pl.CPP * pl.KP * batch <= device_facts().sms;
  auto kern = wide ? gemv_kernel_wide<FMT, NT, EPI, SHAPE> : gemv_kernel<FMT, NT, EPI, SHAPE>;
  cudaError_t e = ensure_smem_attr((const void*)kern, pl.smem_total);
  if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute");
  if (pl.cluster > 1) {
    if (pl.cluster > 8) {
      e = ensure_nonportable_cluster((const void*)kern);
      if (e != cudaSuccess) return check_launch(e, "cudaFuncSetAttribute(non-portable cluster)");
    }
    return check_launch(launch_pdl_cluster(kern, dim3(pl.CPP, pl.KP, (unsigned)batch), dim3(kThreads), pl.smem_total,
                                           st, pl.cluster, a),
                        "gemv cluster launch");
  }
  return check_launch(launch_pdl(kern, dim3(pl.CPP, pl.KP, (unsigned)batch), dim3(kThreads), pl.smem_total, st, a),
                      "gemv launch");
}

template <int FMT, int NT, int EPI>
int launch_t(const Plan& pl, const GemvArgs& a, int64_t batch, cudaStream_t st) {
  if (pl.BI0 == 128) {
    if (pl.NB0 == 2) return launch_s<FMT, NT, EPI, SHAPE_128x2>(pl, a, batch, st);
    return launch_s<FMT, NT, EPI, SHAPE_128x1>(pl, a, batch, st);
  }
  return launch_s<FMT, NT, EPI, SHAPE_64x1>(pl, a, batch, st);
}

template <int FMT, int EPI>
int launch_nt(const Plan& pl, const GemvArgs& a, int64_t batch, cudaStream_t st) {
  return pl.NT == 1 ? launch_t<FMT, 1, EPI>(pl, a, batch, st) : launch_t<FMT, 2, EPI>(pl, a, batch, st);
}


// every (format, epilogue) pair the library launches, instantiated in fp4x_inst_*.cu
extern template int launch_nt<FMT_MX8, EPI_STORE>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_W8, EPI_STORE>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_W8, EPI_HC_DOWN>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_W8, EPI_HC_UP>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_W6, EPI_STORE>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_NV4, EPI_STORE>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_BF16, EPI_STORE>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);
extern template int launch_nt<FMT_INT2, EPI_HEAD>(const Plan&, const GemvArgs&, int64_t, cudaStream_t);

}  // namespace fp4x
