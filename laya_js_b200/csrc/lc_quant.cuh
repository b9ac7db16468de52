// Device helpers for packed 4/8-bit weights (laya-js quantized layout,
// packages/tensor-backend/src/index.ts:98-108; unpacking rule of
// packages/tensor-backend/src/host.ts:155-171).
#pragma once
#include "lc_common.cuh"

// Integer value j of a packed row: 8-bit one byte per value; 4-bit the even
// column in the low nibble. Symmetric values are two's complement.
__device__ __forceinline__ int quant_value(const uint8_t* row, int64_t j, int bits, int mode) {
  if (bits == 8) {
    uint8_t v = row[j];
    return mode == 0 ? (int)(int8_t)v : (int)v;
  }
  uint8_t byte = row[j >> 1];
  int nib = (j & 1) ? (byte >> 4) : (byte & 15);
  return mode == 0 ? ((nib ^ 8) - 8) : nib;
}

// fl(q·s + b) in f64 — exact product, one rounding at the add — then rounded
// once more to the target dtype, exactly as the reference host dequantiser
// computes it in JS doubles and stores into a Float32Array / Float16Array
// (packages/laya/src/quant.ts:199-243).
__device__ __forceinline__ double dequant_f64(int q, float s, float b) { return fma((double)q, (double)s, (double)b); }

__device__ __forceinline__ void store_dequant(char* out, int odt, int64_t i, int q, float s, float b) {
  double v = dequant_f64(q, s, b);
  switch (odt) {
    case LC_F16: ((__half*)out)[i] = __double2half(v); break;
    case LC_BF16: ((__nv_bfloat16*)out)[i] = __double2bfloat16(v); break;
    case LC_F64: ((double*)out)[i] = v; break;
    default: ((float*)out)[i] = (float)v; break;
  }
}

// The dequantised value rounded to `dt`, returned as f32.
__device__ __forceinline__ float dequant_rounded(int dt, int q, float s, float b) {
  double v = dequant_f64(q, s, b);
  switch (dt) {
    case LC_F16: return __half2float(__double2half(v));
    case LC_BF16: return __bfloat162float(__double2bfloat16(v));
    default: return (float)v;
  }
}
