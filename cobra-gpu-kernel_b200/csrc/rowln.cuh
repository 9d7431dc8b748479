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

#include "common.cuh"

namespace b200l {

// VPL = float4 vectors per lane; the row width d must satisfy d <= 128 * VPL.
template <int VPL, bool OUT_F16>
__global__ void __launch_bounds__(256) row_ln_kernel(const float* __restrict__ in, void* __restrict__ out,
                                                     const float* __restrict__ w, const float* __restrict__ b,
                                                     float eps, long long T, int d,
                                                     const uint8_t* __restrict__ rowmask) {
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

// Test hook: arms a fault-injection site and a per-wait time limit in a
// workspace's status block (read by every kernel at its start).
__global__ void debug_arm_kernel(DevStatus* st, int site, unsigned long long wait_ns) {
  st->dbg_site = site;
  st->dbg_wait_ns = wait_ns;
}

}  // namespace b200l
