// Weight preparation on the GPU: the packed formats the decode GEMVs read, produced from fp32 / bf16 / f16 weights
// with the reference's arithmetic (x/fp4x_kernels.py, cited K:<line>), and the dequantizers back to fp32.
//
// The reference quantizers are torch code, and torch evaluates `tensor / python_scalar` differently by device: on
// the CPU it divides, on CUDA it multiplies by the fp32 reciprocal of the scalar.  The two can round a group scale
// one ulp apart, and the packed bytes then differ.  Every quantizer here takes a division mode: FP4X_DIV_IEEE
// reproduces the reference run on the CPU (the committed golden fixtures), FP4X_DIV_RECIP the reference run on a
// CUDA device (what a deployment that quantizes GPU-resident weights produces).  Tensor-by-tensor divisions are IEEE
// divisions in both.
//
// One thread handles one scale group (16, 32 or 64 consecutive weights of a row); these are one-time passes over
// the weights, bound by DRAM like the GEMVs but not on the decode path.
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include <cstring>
#include <string>

#include "fp4x_common.cuh"
#include "fp4x_host.h"

namespace fp4x {

namespace {

constexpr int kPrepThreads = 256;

FP4X_DEV float load_w(const void* w, int dtype, int64_t i) {
  if (dtype == FP4X_IN_F32) return reinterpret_cast<const float*>(w)[i];
  if (dtype == FP4X_IN_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w)[i]);
  return __half2float(reinterpret_cast<const __half*>(w)[i]);
}

// value / scalar as torch computes it on the device the mode names (IEEE division, or the fp32 reciprocal of the
// scalar, rounded once, times the value)
FP4X_DEV float div_scalar(float v, float scalar, float recip, int mode) {
  return mode == FP4X_DIV_RECIP ? v * recip : __fdiv_rn(v, scalar);
}

FP4X_DEV uint32_t f32_to_e4m3_byte(float v) {
  // round to nearest even; the callers clamp to [2^-9, 448] first, so no value saturates
  return (uint32_t)__nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
}

// ---------------------------------------------------------------------------------------------------------------
// W8 g64 (K:138-144): s = max(amax, 1e-12) / 127; q = clamp(round(w / s), -127, 127)
// ---------------------------------------------------------------------------------------------------------------
__global__ void quantize_w8_kernel(const void* w, int dtype, int64_t n, int64_t k, int8_t* q, float* s, int mode) {
  const int64_t groups = n * (k / 64);
  const float r127 = 1.0f / 127.0f;
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t base = gi * 64;
    float amax = 0.f;
    for (int i = 0; i < 64; ++i) amax = fmaxf(amax, fabsf(load_w(w, dtype, base + i)));
    const float sc = div_scalar(fmaxf(amax, 1e-12f), 127.0f, r127, mode);
    s[gi] = sc;
    for (int i = 0; i < 64; ++i) {
      float r = rintf(__fdiv_rn(load_w(w, dtype, base + i), sc));
      r = fminf(fmaxf(r, -127.f), 127.f);
      q[base + i] = (int8_t)r;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// W6 g32 (K:179-202, clip_search = 0): s = max(f32(f16(amax / qmax)), 6.2e-5); q = clamp(round(w / s), -qmax-1,
// qmax) + 32; planes L (nibbles, low = even k) and H (bit pairs in ORDER (0, 2, 1, 3)); S = f16(s)
// ---------------------------------------------------------------------------------------------------------------
__global__ void quantize_w6_kernel(const void* w, int dtype, int64_t n, int64_t k, int qmax, uint8_t* L, uint8_t* H,
                                   __half* S, int mode) {
  const int64_t groups = n * (k / 32);
  const float fq = (float)qmax, rq = 1.0f / (float)qmax;
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t base = gi * 32;
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(load_w(w, dtype, base + i)));
    const float sc = fmaxf(__half2float(__float2half_rn(div_scalar(amax, fq, rq, mode))), 6.2e-5f);
    S[gi] = __float2half_rn(sc);
    int c[32];
    for (int i = 0; i < 32; ++i) {
      float r = rintf(__fdiv_rn(load_w(w, dtype, base + i), sc));
      r = fminf(fmaxf(r, (float)(-qmax - 1)), fq);
      c[i] = (int)r + 32;
    }
    uint8_t* lo = L + base / 2;
    for (int j = 0; j < 16; ++j) lo[j] = (uint8_t)((c[2 * j] & 15) | ((c[2 * j + 1] & 15) << 4));
    uint8_t* hi = H + base / 4;
    for (int j = 0; j < 8; ++j) {
      const int* e = c + 4 * j;
      hi[j] = (uint8_t)((e[0] >> 4) | ((e[2] >> 4) << 2) | ((e[1] >> 4) << 4) | ((e[3] >> 4) << 6));
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// NVFP4 (K:277-300): block scale e4m3(clamp(amax16 / 6 / gs, 2^-9, 448)); v = clamp(w / (f32(scale) * gs), -6, 6);
// magnitude index = number of e2m1 midpoints strictly below |v| (bucketize, ties to the lower magnitude)
// ---------------------------------------------------------------------------------------------------------------
__global__ void amax_kernel(const void* w, int dtype, int64_t count, unsigned int* out) {
  float m = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    m = fmaxf(m, fabsf(load_w(w, dtype, i)));
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) atomicMax(out, __float_as_uint(m));  // non-negative floats order like their bits
}

__global__ void quantize_nv4_kernel(const void* w, int dtype, int64_t n, int64_t k, float gs, float rgs, uint8_t* P,
                                    uint8_t* S, int mode) {
  const int64_t groups = n * (k / 16);
  const float r6 = 1.0f / 6.0f;
  const float mids[7] = {0.25f, 0.75f, 1.25f, 1.75f, 2.5f, 3.5f, 5.0f};
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t base = gi * 16;
    float amax = 0.f;
    for (int i = 0; i < 16; ++i) amax = fmaxf(amax, fabsf(load_w(w, dtype, base + i)));
    float sc = div_scalar(div_scalar(amax, 6.0f, r6, mode), gs, rgs, mode);
    sc = fminf(fmaxf(sc, 0.001953125f), 448.f);
    const uint32_t sb = f32_to_e4m3_byte(sc);
    S[gi] = (uint8_t)sb;
    const float sf = e4m3_to_f32(sb) * gs;
    uint32_t codes[16];
    for (int i = 0; i < 16; ++i) {
      const float v = fminf(fmaxf(__fdiv_rn(load_w(w, dtype, base + i), sf), -6.f), 6.f);
      const float a = fabsf(v);
      uint32_t mag = 0;
      for (int j = 0; j < 7; ++j) mag += a > mids[j] ? 1u : 0u;
      codes[i] = mag | (v < 0.f ? 8u : 0u);
    }
    uint8_t* p = P + base / 2;
    for (int j = 0; j < 8; ++j) p[j] = (uint8_t)(codes[2 * j] | (codes[2 * j + 1] << 4));
  }
}

// ---------------------------------------------------------------------------------------------------------------
// INT2 (K:330-351, fp16 scales): s = f16(max(amax, 1e-8) / 1.5); code = clamp(floor(w / f32(s)) + 2, 0, 3), four
// codes per byte in bit pairs ORDER (0, 2, 1, 3)
// ---------------------------------------------------------------------------------------------------------------
__global__ void quantize_int2_kernel(const void* w, int dtype, int64_t n, int64_t k, int group, uint8_t* P, __half* S,
                                     int mode) {
  const int64_t groups = n * (k / group);
  const float r15 = 1.0f / 1.5f;
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t base = gi * group;
    float amax = 0.f;
    for (int i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(load_w(w, dtype, base + i)));
    const __half sh = __float2half_rn(div_scalar(fmaxf(amax, 1e-8f), 1.5f, r15, mode));
    S[gi] = sh;
    const float sf = __half2float(sh);
    for (int j = 0; j < group / 4; ++j) {
      uint32_t b = 0;
      for (int t = 0; t < 4; ++t) {
        float c = floorf(__fdiv_rn(load_w(w, dtype, base + 4 * j + t), sf)) + 2.f;
        c = fminf(fmaxf(c, 0.f), 3.f);
        const int pos = t == 1 ? 2 : (t == 2 ? 1 : t);
        b |= (uint32_t)c << (2 * pos);
      }
      P[base / 4 + j] = (uint8_t)b;
    }
  }
}

// ---------------------------------------------------------------------------------------------------------------
// dequantizers (fp32 out): MXFP8 K:261-267, NVFP4 K:420-426, INT2 K:353-357
// ---------------------------------------------------------------------------------------------------------------
__global__ void mx8_dequant_kernel(const uint8_t* w8, const uint8_t* s, int64_t n, int64_t k, float* out) {
  const int64_t count = n * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = e4m3_to_f32(w8[i]) * e8m0_to_f32(s[i / 32]);
}

__global__ void dequant_nv4_kernel(const uint8_t* P, const uint8_t* S, float gs, int64_t n, int64_t k, float* out) {
  const float lut[8] = {0.f, 0.5f, 1.f, 1.5f, 2.f, 3.f, 4.f, 6.f};
  const int64_t count = n * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t code = (P[i / 2] >> (4 * (i & 1))) & 15u;
    const float v = (code & 8u) ? -lut[code & 7u] : lut[code & 7u];
    out[i] = v * e4m3_to_f32(S[i / 16]) * gs;
  }
}

__global__ void dequant_int2_kernel(const uint8_t* P, const __half* S, int group, int64_t n, int64_t k, float* out) {
  const int64_t count = n * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i & 3);
    const int pos = t == 1 ? 2 : (t == 2 ? 1 : t);
    const uint32_t c = (P[i / 4] >> (2 * pos)) & 3u;
    out[i] = ((float)c - 1.5f) * __half2float(S[i / group]);
  }
}

// NVFP4 scale tiles of 128 rows x 4 scale columns stored swizzled (the layout of the draft head's source scales,
// x/fp4patch.py:296): swizzled [n/128][kb/4][32][4][4] -> linear [n][kb] with row 128a + 32d + c, column 4b + e
__global__ void nv4_unswizzle_kernel(const uint8_t* in, int64_t n, int64_t kb, uint8_t* out) {
  const int64_t count = n * kb;
  const int64_t kb4 = kb / 4;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < count; o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = o / kb, col = o - row * kb;
    const int64_t a = row / 128, d = (row / 32) & 3, c = row & 31, b = col / 4, e = col & 3;
    out[o] = in[(((a * kb4 + b) * 32 + c) * 4 + d) * 4 + e];
  }
}

// HCFused.interleave_up's row order (K:513-517): out row (j * hc + s) * bj + t = in row s * h + j * bj + t
__global__ void interleave_rows_kernel(const uint8_t* in, int64_t row_bytes, int64_t n, int64_t hc, int64_t bj,
                                       uint8_t* out) {
  const int64_t h = n / hc;
  const int64_t count = n * row_bytes;
  for (int64_t o = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; o < count; o += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = o / row_bytes, byte = o - r * row_bytes;
    const int64_t t = r % bj, js = r / bj, s = js % hc, j = js / hc;
    out[o] = in[(s * h + j * bj + t) * row_bytes + byte];
  }
}

unsigned grid_for(int64_t items) {
  int64_t b = (items + kPrepThreads - 1) / kPrepThreads;
  const int64_t cap = (int64_t)device_facts().sms * 16;
  if (b > cap) b = cap;
  return (unsigned)(b < 1 ? 1 : b);
}

int check_common(const void* w, int dtype, int64_t n, int64_t k, int mode, int kmul) {
  if (!w) return fail(FP4X_ERR_INVALID_ARG, "null weights");
  if (dtype != FP4X_IN_F32 && dtype != FP4X_IN_BF16 && dtype != FP4X_IN_F16)
    return fail(FP4X_ERR_INVALID_ARG, "bad input dtype");
  if (mode != FP4X_DIV_IEEE && mode != FP4X_DIV_RECIP) return fail(FP4X_ERR_INVALID_ARG, "bad division mode");
  if (n < 1 || k < 1 || k % kmul) return fail(FP4X_ERR_UNSUPPORTED, "K must be a multiple of " + std::to_string(kmul));
  return FP4X_OK;
}

int launched(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return check_launch(cudaGetLastError(), what);
}

}  // namespace
}  // namespace fp4x

using namespace fp4x;

extern "C" {

int fp4x_quantize_w8(const void* w, int in_dtype, int64_t n, int64_t k, int8_t* q, float* s, int div_mode,
                     void* stream) {
  int rc = check_common(w, in_dtype, n, k, div_mode, 64);
  if (rc) return rc;
  if (!q || !s) return fail(FP4X_ERR_INVALID_ARG, "null output");
  quantize_w8_kernel<<<grid_for(n * (k / 64)), kPrepThreads, 0, (cudaStream_t)stream>>>(w, in_dtype, n, k, q, s,
                                                                                        div_mode);
  return launched("quantize_w8");
}

int fp4x_quantize_w6(const void* w, int in_dtype, int64_t n, int64_t k, int qmax, uint8_t* lo, uint8_t* hi,
                     void* s_f16, int div_mode, void* stream) {
  int rc = check_common(w, in_dtype, n, k, div_mode, 32);
  if (rc) return rc;
  if (!lo || !hi || !s_f16) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (qmax < 1 || qmax > 31) return fail(FP4X_ERR_INVALID_ARG, "qmax must be in 1..31");
  quantize_w6_kernel<<<grid_for(n * (k / 32)), kPrepThreads, 0, (cudaStream_t)stream>>>(
      w, in_dtype, n, k, qmax, lo, hi, (__half*)s_f16, div_mode);
  return launched("quantize_w6");
}

int fp4x_amax(const void* w, int in_dtype, int64_t count, float* amax_out, void* stream) {
  if (!w || !amax_out || count < 1) return fail(FP4X_ERR_INVALID_ARG, "bad argument");
  if (in_dtype != FP4X_IN_F32 && in_dtype != FP4X_IN_BF16 && in_dtype != FP4X_IN_F16)
    return fail(FP4X_ERR_INVALID_ARG, "bad input dtype");
  cudaError_t e = cudaMemsetAsync(amax_out, 0, sizeof(float), (cudaStream_t)stream);
  if (e != cudaSuccess) return check_launch(e, "amax init");
  amax_kernel<<<grid_for(count), kPrepThreads, 0, (cudaStream_t)stream>>>(w, in_dtype, count, (unsigned int*)amax_out);
  return launched("amax");
}

int fp4x_quantize_nv4(const void* w, int in_dtype, int64_t n, int64_t k, double gs, uint8_t* p, uint8_t* s,
                      int div_mode, void* stream) {
  int rc = check_common(w, in_dtype, n, k, div_mode, 16);
  if (rc) return rc;
  if (!p || !s) return fail(FP4X_ERR_INVALID_ARG, "null output");
  if (!(gs > 0.0)) return fail(FP4X_ERR_INVALID_ARG, "global scale must be positive");
  const float g = (float)gs;  // torch casts the Python scalar to the tensor's fp32
  quantize_nv4_kernel<<<grid_for(n * (k / 16)), kPrepThreads, 0, (cudaStream_t)stream>>>(w, in_dtype, n, k, g,
                                                                                        1.0f / g, p, s, div_mode);
  return launched("quantize_nv4");
}

int fp4x_quantize_int2(const void* w, int in_dtype, int64_t n, int64_t k, int group, uint8_t* p, void* s_f16,
                       int div_mode, void* stream) {
  if (group != 16 && group != 32) return fail(FP4X_ERR_UNSUPPORTED, "INT2 group must be 16 or 32");
  int rc = check_common(w, in_dtype, n, k, div_mode, group);
  if (rc) return rc;
  if (!p || !s_f16) return fail(FP4X_ERR_INVALID_ARG, "null output");
  quantize_int2_kernel<<<grid_for(n * (k / group)), kPrepThreads, 0, (cudaStream_t)stream>>>(
      w, in_dtype, n, k, group, p, (__half*)s_f16, div_mode);
  return launched("quantize_int2");
}

int fp4x_mx8_dequant(const uint8_t* w8, const uint8_t* s, int64_t n, int64_t k, float* out, void* stream) {
  if (!w8 || !s || !out || n < 1 || k < 32 || k % 32) return fail(FP4X_ERR_INVALID_ARG, "bad argument");
  mx8_dequant_kernel<<<grid_for(n * k), kPrepThreads, 0, (cudaStream_t)stream>>>(w8, s, n, k, out);
  return launched("mx8_dequant");
}

int fp4x_dequant_nv4(const uint8_t* p, const uint8_t* s, double gs, int64_t n, int64_t k, float* out, void* stream) {
  if (!p || !s || !out || n < 1 || k < 16 || k % 16) return fail(FP4X_ERR_INVALID_ARG, "bad argument");
  dequant_nv4_kernel<<<grid_for(n * k), kPrepThreads, 0, (cudaStream_t)stream>>>(p, s, (float)gs, n, k, out);
  return launched("dequant_nv4");
}

int fp4x_dequant_int2(const uint8_t* p, const void* s_f16, int group, int64_t n, int64_t k, float* out, void* stream) {
  if (!p || !s_f16 || !out || n < 1 || (group != 16 && group != 32) || k % group)
    return fail(FP4X_ERR_INVALID_ARG, "bad argument");
  dequant_int2_kernel<<<grid_for(n * k), kPrepThreads, 0, (cudaStream_t)stream>>>(p, (const __half*)s_f16, group, n, k,
                                                                                 out);
  return launched("dequant_int2");
}

int fp4x_nv4_unswizzle_scales(const uint8_t* in, int64_t n, int64_t kb, uint8_t* out, void* stream) {
  if (!in || !out || n < 128 || n % 128 || kb < 4 || kb % 4)
    return fail(FP4X_ERR_UNSUPPORTED, "swizzled scales need rows a multiple of 128 and columns a multiple of 4");
  nv4_unswizzle_kernel<<<grid_for(n * kb), kPrepThreads, 0, (cudaStream_t)stream>>>(in, n, kb, out);
  return launched("nv4_unswizzle");
}

int fp4x_interleave_rows(const void* in, int64_t row_bytes, int64_t n, int64_t hc, int64_t bj, void* out,
                         void* stream) {
  if (!in || !out || row_bytes < 1 || hc < 1 || bj < 1 || n % (hc * bj))
    return fail(FP4X_ERR_INVALID_ARG, "rows must be a multiple of hc * bj");
  interleave_rows_kernel<<<grid_for(n * row_bytes), kPrepThreads, 0, (cudaStream_t)stream>>>(
      (const uint8_t*)in, row_bytes, n, hc, bj, (uint8_t*)out);
  return launched("interleave_rows");
}

}  // extern "C"
