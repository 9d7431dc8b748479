// rowln.cuh -- row LayerNorm passes and the weight packer.
//
// Row LayerNorm restates nn.LayerNorm as the reference applies it
// (torch_transformer_benchmark.py:129-131, fused forms :491-535, :450-463):
// biased variance over the row, y = (x - mean) * rsqrt(var + eps) * w + b,
// statistics in fp32. One warp per row, coalesced float4 traffic, the row kept
// in registers between the mean and variance passes (two-pass variance).
// These passes are used where a GEMM epilogue cannot see a whole row
// (d_model > 256), for the block's LN2 (whose fp32 input, the residual, is
// kept for the FFN) and for the stack's final_norm; a row mask zeroes padded
// rows of the output (:170-172).
#pragma once

#include <cuda_bf16.h>

#include "common.cuh"

namespace b200l {

// VPL = float4 vectors per lane; the row width d must satisfy d <= 128 * VPL.
template <int VPL, bool OUT_F16>
__global__ void __launch_bounds__(256) row_ln_kernel(const float* __restrict__ in, void* __restrict__ out,
                                                     const float* __restrict__ w, const float* __restrict__ b,
                                                     float eps, long long T, int d,
                                                     const uint8_t* __restrict__ rowmask) {
  pdl_wait_then_release();
  const int warps = blockDim.x >> 5;
  const long long row = (long long)blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= T) return;
  const bool zero = rowmask != nullptr && rowmask[row] == 0;
  const float* src = in + row * d;
  float4 v[VPL];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 4;
    if (c < d) {
      v[i] = __ldg(reinterpret_cast<const float4*>(src + c));
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    } else {
      v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  const float inv_d = 1.0f / (float)d;
  const float mean = warp_sum(s) * inv_d;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 4;
    if (c < d) {
      const float a = v[i].x - mean, bb = v[i].y - mean, cc = v[i].z - mean, dd = v[i].w - mean;
      q += (a * a + bb * bb) + (cc * cc + dd * dd);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int c = (lane + 32 * i) * 4;
    if (c < d) {
      const float4 ww = __ldg(reinterpret_cast<const float4*>(w + c));
      const float4 bb = __ldg(reinterpret_cast<const float4*>(b + c));
      float4 y;
      y.x = (v[i].x - mean) * rstd * ww.x + bb.x;
      y.y = (v[i].y - mean) * rstd * ww.y + bb.y;
      y.z = (v[i].z - mean) * rstd * ww.z + bb.z;
      y.w = (v[i].w - mean) * rstd * ww.w + bb.w;
      if (zero) y = make_float4(0.f, 0.f, 0.f, 0.f);
      if constexpr (OUT_F16) {
        uint2 p;
        p.x = pack_half2(y.x, y.y);
        p.y = pack_half2(y.z, y.w);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(out) + row * d + c) = p;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + row * d + c) = y;
      }
    }
  }
}

// wqkv16[3d, d] = fp16(cat(wq, wk, wv)), bqkv32 = cat(bq, bk, bv), wo16 = fp16(wo).
__global__ void pack_weights_kernel(int d, const float* __restrict__ wq, const float* __restrict__ wk,
                                    const float* __restrict__ wv, const float* __restrict__ bq,
                                    const float* __restrict__ bk, const float* __restrict__ bv,
                                    const float* __restrict__ wo, __half* __restrict__ wqkv16,
                                    float* __restrict__ bqkv32, __half* __restrict__ wo16) {
  const long long dd = (long long)d * d;
  const long long total = 4 * dd;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int which = (int)(i / dd);
    const long long off = i - which * dd;
    if (which < 3) {
      const float* src = which == 0 ? wq : (which == 1 ? wk : wv);
      wqkv16[i] = __float2half_rn(src[off]);
    } else {
      wo16[off] = __float2half_rn(wo[off]);
    }
    if (i < 3LL * d) {
      const int w2 = (int)(i / d);
      const float* bsrc = w2 == 0 ? bq : (w2 == 1 ? bk : bv);
      bqkv32[i] = bsrc[i - (long long)w2 * d];
    }
  }
}

// dst[i] = fp16(src[i]): weight packing for the FFN matrices.
__global__ void cast_f16_kernel(const float* __restrict__ src, __half* __restrict__ dst, long long n) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    dst[i] = __float2half_rn(src[i]);
}

// dst = src converted between fp32 / fp16 / bf16 (round to nearest even),
// eight elements per thread and step (16-byte fp16 / bf16 accesses): the
// boundary conversion for reduced-precision inputs and outputs.
enum ElemType : int { kF32 = 0, kF16 = 1, kBF16 = 2 };

template <int SRC, int DST>
__global__ void convert_kernel(const void* __restrict__ src, void* __restrict__ dst, long long n) {
  const long long n8 = n / 8;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8 + (n % 8 ? 1 : 0); i += stride) {
    float v[8];
    const long long e0 = i * 8;
    const int cnt = (e0 + 8 <= n) ? 8 : (int)(n - e0);
    if (cnt == 8) {
      if constexpr (SRC == kF32) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(src) + 2 * i);
        const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 2 * i + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
      } else {
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(src) + i);
        const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 f;
          if constexpr (SRC == kF16) f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
          else f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[k]));
          v[2 * k] = f.x; v[2 * k + 1] = f.y;
        }
      }
    } else {
      for (int k = 0; k < cnt; ++k) {
        if constexpr (SRC == kF32) v[k] = reinterpret_cast<const float*>(src)[e0 + k];
        else if constexpr (SRC == kF16) v[k] = __half2float(reinterpret_cast<const __half*>(src)[e0 + k]);
        else v[k] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(src)[e0 + k]);
      }
    }
    if (cnt == 8) {
      if constexpr (DST == kF32) {
        reinterpret_cast<float4*>(dst)[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(dst)[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
      } else {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if constexpr (DST == kF16) {
            const __half2 h = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
            w[k] = *reinterpret_cast<const uint32_t*>(&h);
          } else {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * k], v[2 * k + 1]);
            w[k] = *reinterpret_cast<const uint32_t*>(&h);
          }
        }
        reinterpret_cast<uint4*>(dst)[i] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
      for (int k = 0; k < cnt; ++k) {
        if constexpr (DST == kF32) reinterpret_cast<float*>(dst)[e0 + k] = v[k];
        else if constexpr (DST == kF16) reinterpret_cast<__half*>(dst)[e0 + k] = __float2half_rn(v[k]);
        else reinterpret_cast<__nv_bfloat16*>(dst)[e0 + k] = __float2bfloat16_rn(v[k]);
      }
    }
  }
}

// Test hook: arms a fault-injection site and a per-wait time limit in a
// workspace's status block (read by every kernel at its start).
__global__ void debug_arm_kernel(DevStatus* st, int site, unsigned long long wait_ns) {
  st->dbg_site = site;
  st->dbg_wait_ns = wait_ns;
}

}  // namespace b200l
