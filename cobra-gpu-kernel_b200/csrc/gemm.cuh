// gemm.cuh -- tcgen05 GEMMs of the layer: K1 (LayerNorm-fused QKV projection)
// and the TMA-fed GEMM used for the out-projection (K3, with the residual +
// LayerNorm epilogue) and for the QKV projection when d_model > 256.
//
// Both compute D[128 x N] = A[128 x K] * B[N x K]^T with fp16 operands in
// shared memory (K-major, 128-byte swizzle) and fp32 accumulators in TMEM,
// issued by one thread (tcgen05.mma.cta_group::1.kind::f16, M = 128).
// Thread-per-row epilogues: warp w reads TMEM lanes 32*(w%4)..+31, so each
// thread owns one output row and row reductions need no shuffles.
//
// Reference counterparts: _gemm_kernel (torch_transformer_benchmark.py:283-353),
// _gemm_ln_kernel (:394-463), _add_ln_kernel (:491-535, as used at :1220-1223).
#pragma once

#include "common.cuh"

namespace b200l {

// Destination of the QKV projection: q, k as [B*H, S, dhp] and v transposed as
// [B*H, dhp, sp] (sp = S rounded up to 8, so every row stride is 16-byte
// aligned for TMA), all fp16. Columns dh..dhp-1 are written as zeros.
struct QkvOut {
  __half* q;
  __half* k;
  __half* vt;
  int S, H, dh, dhp, sp;
  int dq;   // width of each of the q / k / v projections: H * dh (the heads computed)
};

// Tensor maps of the q, k (fp16 [B*H, S, dhp]) and v^T (fp16 [B*H, dhp, sp])
// outputs in 32 x 32 boxes with the 64-byte swizzle, for the QKV epilogue's
// TMA stores; `use` is 0 when they are not set (the per-thread stores run).
struct alignas(64) QkvMaps {
  CUtensorMap q, k, vt;
  int use;
};

// Stores 32 consecutive projection columns [col0, col0+32) of token t.
// dh is a multiple of 32, so the chunk lies inside one (q|k|v, head) block.
__device__ __forceinline__ void qkv_store_chunk(const QkvOut& o, const float* __restrict__ bqkv, long long t,
                                                int col0, const uint32_t (&acc)[32]) {
  const int which = col0 / o.dq;
  const int within = col0 - which * o.dq;
  const int head = within / o.dh;
  const int j0 = within - head * o.dh;
  const long long b = t / o.S;
  const int s = (int)(t - b * o.S);
  const long long bh = b * o.H + head;
  float v[32];
#pragma unroll
  for (int i = 0; i < 8; ++i) {   // bqkv is 16-byte aligned (checked on the host), col0 % 32 == 0
    const float4 b4 = __ldg(reinterpret_cast<const float4*>(bqkv + col0) + i);
    v[4 * i + 0] = __uint_as_float(acc[4 * i + 0]) + b4.x;
    v[4 * i + 1] = __uint_as_float(acc[4 * i + 1]) + b4.y;
    v[4 * i + 2] = __uint_as_float(acc[4 * i + 2]) + b4.z;
    v[4 * i + 3] = __uint_as_float(acc[4 * i + 3]) + b4.w;
  }
  const bool pad_tail = (j0 + 32 == o.dh) && (o.dhp > o.dh);
  if (which < 2) {
    __half* dst = (which == 0 ? o.q : o.k) + (bh * o.S + s) * (long long)o.dhp + j0;
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      d4[c] = make_uint4(pack_half2(v[8 * c + 0], v[8 * c + 1]), pack_half2(v[8 * c + 2], v[8 * c + 3]),
                         pack_half2(v[8 * c + 4], v[8 * c + 5]), pack_half2(v[8 * c + 6], v[8 * c + 7]));
    }
    if (pad_tail) {
      uint4* z = reinterpret_cast<uint4*>(dst + 32);
      for (int c = 0; c < (o.dhp - o.dh) / 8; ++c) z[c] = make_uint4(0, 0, 0, 0);
    }
  } else {
    __half* dst = o.vt + (bh * o.dhp + j0) * (long long)o.sp + s;
#pragma unroll
    for (int i = 0; i < 32; ++i) dst[(long long)i * o.sp] = __float2half_rn(v[i]);
    if (pad_tail) {
      for (int jj = 32; jj < 32 + (o.dhp - o.dh); ++jj) dst[(long long)jj * o.sp] = __float2half_rn(0.f);
    }
  }
}

// ===========================================================================
// K1: h = LN1(x) -> [q|k|v] = h Wqkv^T + bqkv, for d_model <= 256.
//
// One CTA per 128-token block. All 8 warps normalise the block's rows (warp
// per row, coalesced fp32 loads, two-pass variance) straight into the fp16
// A operand in shared memory, where it stays for every N tile, so x is read
// exactly once and h never touches HBM. Weight tiles [128 x KP] stream in by
// TMA (2 stages); accumulators are double-buffered in TMEM (2 x 128 columns)
// so the epilogue of tile n overlaps the MMAs of tile n+1.
// KP = d rounded up to 64 (the padding columns of A are written as zeros and
// the weight map's out-of-range columns are zero-filled by TMA).
// ===========================================================================
template <int KP>
struct QkvLnFusedCfg {
  static constexpr int KC = KP / 64;                // 128-byte atom columns
  static constexpr int A_BYTES = KC * 128 * 128;    // 128 rows
  static constexpr int W_BYTES = KC * 128 * 128;    // one 128-row N tile
  static constexpr int WST = 2;
  static constexpr int SMEM = A_BYTES + WST * W_BYTES + 256 + 1024;  // + barriers + alignment slack
  static constexpr int NV = (KP + 127) / 128;       // float4 per lane in the LN prologue
};

template <int KP>
__global__ void __launch_bounds__(256, 1)
    qkv_lnfused_kernel(const __grid_constant__ CUtensorMap map_w, const float* __restrict__ x,
                       const float* __restrict__ ln_w, const float* __restrict__ ln_b, float eps,
                       const float* __restrict__ bqkv, QkvOut out, long long T, int d, int N, DevStatus* status) {
  pdl_wait_then_release();
  using C = QkvLnFusedCfg<KP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sW = smem + C::A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sW + C::WST * C::W_BYTES);
  uint64_t* w_full = bars;         // [2]
  uint64_t* w_empty = bars + 2;    // [2]
  uint64_t* acc_full = bars + 4;   // [2]
  uint64_t* acc_empty = bars + 6;  // [2]
  uint64_t* mma_done = bars + 8;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);
  WaitCtl* wc = reinterpret_cast<WaitCtl*>(bars + 10);   // bars 10-11

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long long m0 = (long long)blockIdx.x * 128;
  const int NT = (N + 127) / 128;   // N = 3 * out.dq projection columns
  const int KS = (d + 15) / 16;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    waitctl_init(wc, status);
    fence_barrier_init();
    tma_prefetch_desc(&map_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Start the first weight tiles before the LayerNorm prologue.
  const int npro = NT < C::WST ? NT : C::WST;
  if (threadIdx.x == 0) {
    for (int n = 0; n < npro; ++n) {
      mbar_arrive_expect_tx(&w_full[n], C::W_BYTES);
      for (int kc = 0; kc < C::KC; ++kc) tma_load_2d(sW + n * C::W_BYTES + kc * 16384, &map_w, &w_full[n], kc * 64, n * 128);
    }
  }

  // ---- LayerNorm prologue: 16 rows per warp, into the swizzled fp16 A tile.
  // The loads of RB rows are issued together (RB * NV float4 per lane in
  // flight), so a warp waits for memory once per group of rows, not per row.
  {
    constexpr int RB = 16 / C::NV;
    const float inv_d = 1.0f / (float)d;
    const uint32_t a_base = smem_u32(sA);
    float4 w4[C::NV], b4[C::NV];
#pragma unroll
    for (int i = 0; i < C::NV; ++i) {
      const int k = (lane + 32 * i) * 4;
      w4[i] = k < d ? __ldg(reinterpret_cast<const float4*>(ln_w + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
      b4[i] = k < d ? __ldg(reinterpret_cast<const float4*>(ln_b + k)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll 1
    for (int r0 = 0; r0 < 16; r0 += RB) {
      float4 v[RB][C::NV];
#pragma unroll
      for (int rr = 0; rr < RB; ++rr) {
        const long long t = m0 + warp * 16 + r0 + rr;
#pragma unroll
        for (int i = 0; i < C::NV; ++i) {
          const int k = (lane + 32 * i) * 4;
          v[rr][i] = (t < T && k < d) ? ldg_stream_f4(x + t * d + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int rr = 0; rr < RB; ++rr) {
        const int row = warp * 16 + r0 + rr;
        const bool valid = m0 + row < T;
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < C::NV; ++i) s += (v[rr][i].x + v[rr][i].y) + (v[rr][i].z + v[rr][i].w);
        const float mean = warp_sum(s) * inv_d;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < C::NV; ++i) {
          const int k = (lane + 32 * i) * 4;
          if (k < d) {
            const float a = v[rr][i].x - mean, b = v[rr][i].y - mean, c = v[rr][i].z - mean, e = v[rr][i].w - mean;
            q += (a * a + b * b) + (c * c + e * e);
          }
        }
        const float rstd = rsqrtf(warp_sum(q) * inv_d + eps);
#pragma unroll
        for (int i = 0; i < C::NV; ++i) {
          const int k = (lane + 32 * i) * 4;
          if (k < KP) {
            uint32_t lo = 0, hi = 0;
            if (valid && k < d) {
              lo = pack_half2((v[rr][i].x - mean) * rstd * w4[i].x + b4[i].x,
                              (v[rr][i].y - mean) * rstd * w4[i].y + b4[i].y);
              hi = pack_half2((v[rr][i].z - mean) * rstd * w4[i].z + b4[i].z,
                              (v[rr][i].w - mean) * rstd * w4[i].w + b4[i].w);
            }
            const int kc = k >> 6, kin = k & 63;
            st_shared_v2(a_base + kc * 16384 + swz_offset(row, kin >> 3, 128) + (kin & 7) * 2, lo, hi);
          }
        }
      }
    }
  }
  fence_proxy_async_smem();
  __syncthreads();

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer for the remaining weight tiles
      int last[2] = {-1, -1};
      for (int n = 0; n < npro; ++n) last[n] = n;
      for (int n = C::WST; n < NT; ++n) {
        const int s = n % C::WST;
        if (!mbar_wait(&w_empty[s], ((n / C::WST) & 1) ^ 1, wc)) break;
        mbar_arrive_expect_tx(&w_full[s], C::W_BYTES);
        for (int kc = 0; kc < C::KC; ++kc)
          tma_load_2d(sW + s * C::W_BYTES + kc * 16384, &map_w, &w_full[s], kc * 64, n * 128);
        last[s] = n;
      }
      for (int s = 0; s < 2; ++s)
        if (last[s] >= 0) mbar_drain(&w_full[s], (last[s] / C::WST) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = idesc_f16_f32(128, 128);
      const uint32_t a_base = smem_u32(sA);
      for (int n = 0; n < NT; ++n) {
        const int s = n % C::WST, a = n & 1;
        if (!mbar_wait(&w_full[s], (n / C::WST) & 1, wc)) break;
        if (!mbar_wait(&acc_empty[a], ((n >> 1) & 1) ^ 1, wc)) break;
        tc_fence_after();
        const uint32_t w_base = smem_u32(sW + s * C::W_BYTES);
        for (int k = 0; k < KS; ++k) {
          const uint32_t off = (k >> 2) * 16384 + (k & 3) * 32;
          umma_f16_ss(tmem_base + a * 128, sdesc_kmajor(a_base + off, 128), sdesc_kmajor(w_base + off, 128), idesc,
                      k > 0 ? 1u : 0u);
        }
        umma_commit(&w_empty[s]);
        umma_commit(&acc_full[a]);
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp >= 4) {  // ---- epilogue: bias, fp16, scatter to q / k / v^T
    const int qd = warp & 3;
    const int row = qd * 32 + lane;
    const long long t = m0 + row;
    const bool valid = t < T;
    for (int n = 0; n < NT; ++n) {
      const int a = n & 1;
      if (!mbar_wait(&acc_full[a], (n >> 1) & 1, wc)) break;
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        const int col0 = n * 128 + cc * 32;
        if (col0 >= N) break;
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(qd * 32) << 16) + a * 128 + cc * 32, r);
        if (valid) qkv_store_chunk(out, bqkv, t, col0, r);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && waitctl_aborted(wc)) record_error(status, kErrTimeout, kQkvLnFused, 0);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 256);
  }
}

// ===========================================================================
// TMA-fed GEMM: D[128 x BN] = A[128 x K] * B[BN x K]^T over a ST-stage ring of
// (A 128x64, B BNx64) fp16 tiles. Persistent: each CTA walks output tiles
// (m-major, so neighbouring tiles share A), the producer and the MMA issuer
// run ahead across tile boundaries, and two TMEM accumulators (when 2*BN fits
// in 512 columns) let the epilogue of one tile overlap the MMAs of the next.
// Epilogues:
//   EPI_QKV       bias + scatter into q / k / v^T        (QKV for d > 256)
//   EPI_RESID     y = x + acc + bias  (fp32, pre-LN)      (out-proj for d > 256)
//   EPI_RESID_LN  y = LN2(x + acc + bias), BN >= d        (out-proj for d <= 256)
//   EPI_GELU      h = fp16(gelu_erf(acc + bias))          (FFN in, :142, :326-328)
// The residual is added to the fp32 accumulator and never rounded to fp16
// before the add (the reference's fp32-store rule, :187-191, :350-353).
// Warps: 0 TMA producer, 1 MMA issuer + TMEM owner, 2-5 epilogue.
// ===========================================================================
enum EpiKind : int { EPI_QKV = 0, EPI_RESID = 1, EPI_RESID_LN = 2, EPI_GELU = 3 };

struct EpiArgs {
  QkvOut qkv;
  const float* bias;
  const float* x;
  float* y;
  const float* ln_w;
  const float* ln_b;
  float eps;
  int d;
  const uint8_t* rowmask;  // EPI_RESID*: token validity uint8 [T] or nullptr; invalid rows get y = x (+ LN)
  int rowmask_zero;        // EPI_RESID: invalid rows get y = 0 instead (end of a block, :144-145)
  __half* h;               // EPI_GELU output, fp16 [T, ldh]
  int ldh;
};

// Residual x of one row, columns [col0, col0 + 32), as 8 float4 (zeros past
// lim or for rows beyond T). Issued a chunk ahead of its use, so the HBM
// latency of one chunk overlaps the work on the previous one. The eight loads
// of a thread share one 128-byte line, so they go through L1.
__device__ __forceinline__ void load_x_chunk(const float* xr, int col0, bool valid, int lim, float4 (&v)[8]) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    v[c] = (valid && col0 + 4 * c < lim) ? __ldg(reinterpret_cast<const float4*>(xr + col0 + 4 * c))
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
}

template <int BN, int ST>
struct GemmTmaCfg {
  static constexpr int A_BYTES = 128 * 128;  // 128 rows x 64 fp16
  static constexpr int B_BYTES = BN * 128;   // BN rows x 64 fp16
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int SMEM = ST * STAGE + 256 + 1024;
  static constexpr int QKV_STAGE = 4 * 2 * 2048;       // EPI_QKV: two 32 x 32 fp16 boxes per epilogue warp
  static constexpr int SMEM_QKV = ST * STAGE + 1024 + QKV_STAGE + 1024;
  static constexpr int ACC_COLS = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr int NACC = 2 * ACC_COLS <= 512 ? 2 : 1;      // TMEM accumulators
  static constexpr int TMEM_COLS = NACC * ACC_COLS;
};

template <int BN, int ST, int EPI>
__global__ void __launch_bounds__(192, 1)
    gemm_tma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                    const __grid_constant__ QkvMaps qm, EpiArgs ea, long long T, int K, int N, DevStatus* status) {
  pdl_wait_then_release();
  using C = GemmTmaCfg<BN, ST>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + ST * C::STAGE);
  uint64_t* full = bars;                    // [ST]
  uint64_t* empty = bars + ST;              // [ST]
  uint64_t* acc_full = bars + 2 * ST;       // [NACC]
  uint64_t* acc_empty = bars + 2 * ST + 2;  // [NACC], one arrival per epilogue warp
  uint64_t* mma_done = bars + 2 * ST + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 5);
  WaitCtl* wc = reinterpret_cast<WaitCtl*>(bars + 2 * ST + 6);   // 2 slots

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NT = (N + BN - 1) / BN;
  const long long tiles = ((T + 127) / 128) * NT;
  const int KT = (K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(mma_done, 1);
    waitctl_init(wc, status);
    fence_barrier_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- producer: A/B k-tiles of every tile of this CTA, in order
      int last[ST];
      for (int i = 0; i < ST; ++i) last[i] = -1;
      long long it = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
        const long long m0 = (tile / NT) * 128;
        const int n0 = (int)(tile % NT) * BN;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = (int)(it % ST);
          if (!mbar_wait(&empty[s], (uint32_t)((it / ST) & 1) ^ 1u, wc)) { ok = false; break; }
          // Test hook: CTA 0 leaves out its first operand load (nothing issued,
          // so nothing to drain); the MMA issuer's bounded wait runs out.
          if (it == 0 && blockIdx.x == 0 && wc->site == kSiteGemmOperand) continue;
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          uint8_t* st = smem + s * C::STAGE;
          tma_load_2d(st, &map_a, &full[s], kt * 64, (int)m0);
          tma_load_2d(st + C::A_BYTES, &map_b, &full[s], kt * 64, n0);
          last[s] = (int)(it / ST);
        }
      }
      for (int s = 0; s < ST; ++s)
        if (last[s] >= 0) mbar_drain(&full[s], last[s] & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = idesc_f16_f32(128, BN);
      long long it = 0;
      int ti = 0;
      bool ok = true;
      for (long long tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++ti) {
        const int a = ti % C::NACC;
        const int use = ti / C::NACC;   // earlier tiles that used accumulator a
        if (use > 0 && !mbar_wait(&acc_empty[a], (use - 1) & 1, wc)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * C::ACC_COLS;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = (int)(it % ST);
          if (!mbar_wait(&full[s], (uint32_t)((it / ST) & 1), wc)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * C::STAGE);
          const uint32_t b_base = a_base + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss(d_tmem, sdesc_kmajor(a_base + kk * 32, 128), sdesc_kmajor(b_base + kk * 32, 128), idesc,
                        (kt | kk) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[a]);
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else {  // ---- epilogue warps 2..5, one output row per thread
    const int qd = warp & 3;
    const int row = qd * 32 + lane;
    int ti = 0;
    uint8_t* qstage = smem + ST * C::STAGE + 1024 + (warp - 2) * 4096;   // EPI_QKV staging
    int nqst = 0;
    float4 xn[8];          // EPI_RESID_LN: the next x chunk of this thread's row, loaded ahead
    bool x_next = false;   // xn already holds the first chunk of this tile's row
    for (long long tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++ti) {
      const long long m0 = (tile / NT) * 128;
      const int n0 = (int)(tile % NT) * BN;
      const int a = ti % C::NACC;
      const long long t = m0 + row;
      const bool valid = t < T;
      const uint32_t tl = tmem_base + a * C::ACC_COLS + ((uint32_t)(qd * 32) << 16);
      // EPI_RESID_LN: the row's first x chunk is loaded before the wait for
      // the accumulator (x does not depend on it), or was loaded during the
      // previous tile.
      const float* xrow = ea.x + t * ea.d;
      if constexpr (EPI == EPI_RESID_LN) {
        if (!x_next) load_x_chunk(xrow, 0, valid, ea.d, xn);
        x_next = false;
      }
      if (!mbar_wait_warp(&acc_full[a], (uint32_t)(ti / C::NACC) & 1, wc)) break;
      tc_fence_after();
      if constexpr (EPI == EPI_QKV) {
        // A warp whose 32 rows lie in one sequence stores each 32-column chunk
        // as one 32 x 32 box by TMA (q / k rows, or the transposed v^T block),
        // staged through 64-byte-swizzled shared memory; other warps (a
        // sequence boundary inside the rows, rows past T, padded head_dim)
        // store per thread.
        const QkvOut& o = ea.qkv;
        const long long r0 = m0 + qd * 32;
        const long long b0 = r0 / o.S;
        const int s0 = (int)(r0 - b0 * o.S);
        const bool box_ok = qm.use && r0 + 31 < T && s0 + 31 < o.S && o.dh == o.dhp;
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          const int col0 = n0 + cc * 32;
          if (col0 >= N) break;
          uint32_t r[32];
          tmem_ld32(tl + cc * 32, r);
          const int which = col0 / o.dq;
          if (!box_ok || (which == 2 && (s0 & 7) != 0)) {   // v^T boxes start on a 16-byte column
            if (valid) qkv_store_chunk(o, ea.bias, t, col0, r);
            continue;
          }
          const int within = col0 - which * o.dq;
          const int head = within / o.dh;
          const int j0 = within - head * o.dh;
          const int bh = (int)(b0 * o.H + head);
          uint8_t* yb = qstage + (nqst & 1) * 2048;
          ++nqst;
          if (lane == 0) bulk_wait_read<1>();   // the store that last used this buffer has read it
          __syncwarp();
          const uint32_t ys = smem_u32(yb);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) {   // bqkv is 16-byte aligned (checked on the host)
            const float4 b4 = __ldg(reinterpret_cast<const float4*>(ea.bias + col0) + i);
            pk[2 * i] = pack_half2(__uint_as_float(r[4 * i + 0]) + b4.x, __uint_as_float(r[4 * i + 1]) + b4.y);
            pk[2 * i + 1] = pack_half2(__uint_as_float(r[4 * i + 2]) + b4.z, __uint_as_float(r[4 * i + 3]) + b4.w);
          }
          if (which < 2) {   // this lane's row: four 16-byte pieces
#pragma unroll
            for (int c = 0; c < 4; ++c)
              st_shared_v4(ys + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                           pk[4 * c + 3]);
          } else {           // this lane's token is column `lane` of the 32 (head_dim) x 32 (token) box
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const uint32_t w = pk[jj >> 1];
              st_shared_u16(ys + jj * 64 + (((lane >> 3) ^ ((jj >> 1) & 3)) << 4) + (lane & 7) * 2,
                            (unsigned short)((jj & 1) ? (w >> 16) : (w & 0xffffu)));
            }
          }
          fence_proxy_async_smem();   // generic writes before the async-proxy (TMA) read
          __syncwarp();
          if (lane == 0) {
            if (which == 0) tma_store_3d(&qm.q, yb, j0, s0, bh);
            else if (which == 1) tma_store_3d(&qm.k, yb, j0, s0, bh);
            else tma_store_3d(&qm.vt, yb, s0, j0, bh);
            bulk_commit();
          }
        }
      } else if constexpr (EPI == EPI_RESID) {
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          const int col0 = n0 + cc * 32;
          if (col0 >= N) break;
          uint32_t r[32];
          tmem_ld32(tl + cc * 32, r);
          if (valid) {
            const float* xr = xrow + col0;
            float* yr = ea.y + t * ea.d + col0;
            // A padded query row's attention output is zeroed (bias included):
            // y = x there (BaselineSelfAttention, :121-122); at the end of a
            // block the whole padded row is zeroed instead (:144-145).
            const bool keep = ea.rowmask == nullptr || ea.rowmask[t] != 0;
            const float xs = (!keep && ea.rowmask_zero) ? 0.f : 1.f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const float4 xv = __ldg(reinterpret_cast<const float4*>(xr) + c);
              const float4 bv = __ldg(reinterpret_cast<const float4*>(ea.bias + col0) + c);
              float4 o;
              o.x = xs * xv.x + (keep ? __uint_as_float(r[4 * c + 0]) + bv.x : 0.f);
              o.y = xs * xv.y + (keep ? __uint_as_float(r[4 * c + 1]) + bv.y : 0.f);
              o.z = xs * xv.z + (keep ? __uint_as_float(r[4 * c + 2]) + bv.z : 0.f);
              o.w = xs * xv.w + (keep ? __uint_as_float(r[4 * c + 3]) + bv.w : 0.f);
              reinterpret_cast<float4*>(yr)[c] = o;
            }
          }
        }
      } else if constexpr (EPI == EPI_GELU) {
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          const int col0 = n0 + cc * 32;
          if (col0 >= N) break;
          uint32_t r[32];
          tmem_ld32(tl + cc * 32, r);
          if (valid) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {   // 8 columns -> one 16-byte store
              const int c0 = col0 + 8 * g;
              if (c0 < N) {
                uint32_t w[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float v0 = __uint_as_float(r[8 * g + 2 * e]) + __ldg(ea.bias + c0 + 2 * e);
                  float v1 = __uint_as_float(r[8 * g + 2 * e + 1]) + __ldg(ea.bias + c0 + 2 * e + 1);
                  // exact GELU, F.gelu(approximate="none"): 0.5 v (1 + erf(v / sqrt(2)))
                  v0 = 0.5f * v0 * (1.0f + erff(v0 * 0.70710678118654752f));
                  v1 = 0.5f * v1 * (1.0f + erff(v1 * 0.70710678118654752f));
                  w[e] = pack_half2(v0, v1);
                }
                *reinterpret_cast<uint4*>(ea.h + t * ea.ldh + c0) = make_uint4(w[0], w[1], w[2], w[3]);
              }
            }
          }
        }
      } else {  // EPI_RESID_LN: the whole row is in this tile (n0 == 0, BN >= d)
        const int d = ea.d;
        const bool keep = ea.rowmask == nullptr || (valid && ea.rowmask[t] != 0);  // see EPI_RESID
        float sum = 0.f;
        // pass 1: r = x + (acc + b), written back into TMEM; row sum.
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          float4 xc[8];
#pragma unroll
          for (int c = 0; c < 8; ++c) xc[c] = xn[c];
          if (cc + 1 < BN / 32) {
            load_x_chunk(xrow, cc * 32 + 32, valid, d, xn);
          } else if (tile + gridDim.x < tiles) {   // the next tile's first chunk
            const long long tn = ((tile + gridDim.x) / NT) * 128 + row;
            load_x_chunk(ea.x + tn * d, 0, tn < T, d, xn);
            x_next = true;
          }
          uint32_t r[32];
          tmem_ld32(tl + cc * 32, r);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int col = cc * 32 + 4 * c;
            if (valid && col < d) {
              const float4 xv = xc[c];
              const float4 bv = __ldg(reinterpret_cast<const float4*>(ea.bias + col));
              const float a0 = xv.x + (keep ? __uint_as_float(r[4 * c + 0]) + bv.x : 0.f);
              const float a1 = xv.y + (keep ? __uint_as_float(r[4 * c + 1]) + bv.y : 0.f);
              const float a2 = xv.z + (keep ? __uint_as_float(r[4 * c + 2]) + bv.z : 0.f);
              const float a3 = xv.w + (keep ? __uint_as_float(r[4 * c + 3]) + bv.w : 0.f);
              sum += (a0 + a1) + (a2 + a3);
              r[4 * c + 0] = __float_as_uint(a0);
              r[4 * c + 1] = __float_as_uint(a1);
              r[4 * c + 2] = __float_as_uint(a2);
              r[4 * c + 3] = __float_as_uint(a3);
            }
          }
          tmem_st32(tl + cc * 32, r);
        }
        const float inv_d = 1.0f / (float)d;
        const float mean = sum * inv_d;
        // pass 2: variance about the mean.
        float sq = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(tl + cc * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = cc * 32 + i;
            if (col < d) {
              const float dv = __uint_as_float(r[i]) - mean;
              sq += dv * dv;
            }
          }
        }
        const float rstd = rsqrtf(sq * inv_d + ea.eps);
        // pass 3: normalise and store.
#pragma unroll 1
        for (int cc = 0; cc < BN / 32; ++cc) {
          uint32_t r[32];
          tmem_ld32(tl + cc * 32, r);
          if (valid) {
            float* yr = ea.y + t * d;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int col = cc * 32 + 4 * c;
              if (col < d) {
                const float4 wv = __ldg(reinterpret_cast<const float4*>(ea.ln_w + col));
                const float4 bv = __ldg(reinterpret_cast<const float4*>(ea.ln_b + col));
                float4 o;
                o.x = (__uint_as_float(r[4 * c + 0]) - mean) * rstd * wv.x + bv.x;
                o.y = (__uint_as_float(r[4 * c + 1]) - mean) * rstd * wv.y + bv.y;
                o.z = (__uint_as_float(r[4 * c + 2]) - mean) * rstd * wv.z + bv.z;
                o.w = (__uint_as_float(r[4 * c + 3]) - mean) * rstd * wv.w + bv.w;
                *reinterpret_cast<float4*>(yr + col) = o;
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    if constexpr (EPI == EPI_QKV) {
      if (lane == 0) bulk_wait_all();   // this warp's q / k / v^T box stores are complete
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && waitctl_aborted(wc)) record_error(status, kErrTimeout, kGemmTma, EPI);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

// ===========================================================================
// Out-projection with the residual and LayerNorm-2 in the epilogue for
// d_model = NC * 256 > 256: y = LN2(x + ctx Wo^T + bo).
//
// A 256-column accumulator per CTA cannot see a whole row, so a cluster of NC
// CTAs shares each 128-row M tile, CTA rank r owning output columns
// [256 r, 256 r + 256). Each epilogue thread (one row) forms r = x + acc + bo
// for its 256 columns (written back to TMEM), its mean and the sum of squared
// deviations about it (one pass: sums of the differences from the row's first
// value here and of their squares), stores that pair into every CTA
// of the cluster (distributed shared memory) and arrives on each CTA's stats
// barrier with cluster-scope release. After the cluster-scope acquire, each
// thread combines the NC pairs (equal counts: mean = average of the means,
// M2 = sum of M2 + 256 * sum of squared mean offsets), normalises its 256
// columns from TMEM and stores y. The residual is added in fp32 before any
// rounding, as in EPI_RESID_LN (reference _gemm_ln_kernel,
// torch_transformer_benchmark.py:394-463, which needs the whole row in one
// tile; the reference's fallback for wider rows is a separate _add_ln_kernel
// pass, :1289-1292 -- this kernel removes that pass).
//
// The residual and the output move by TMA, in 32-column chunks of the tile
// (128B-swizzled shared memory, so one thread per row reads and writes
// 16-byte pieces without bank conflicts beyond the minimum):
//   * warp 6 streams x chunks [128 rows x 32] into a two-chunk ring as soon
//     as a slot frees -- x does not depend on the accumulator, so the next
//     tile's first chunks land while this tile is still being normalised, and
//     many bytes are in flight without holding registers;
//   * each epilogue warp writes its 32 rows x 32 normalised columns into one
//     of its two staging buffers and issues a TMA store of that box: full
//     128-byte lines, rows past T clipped by the tensor map.
// Every CTA of a cluster walks the same M tiles (cluster c: tiles c, c +
// nclusters, ...), with the TMA producer and the MMA issuer running ahead
// into the second TMEM accumulator. No TMA load uses cluster multicast: each
// CTA loads its own A tile, its 256 rows of Wo and its x columns.
// Warps: 0 A / B producer, 1 MMA issuer + TMEM owner, 2-5 epilogue, 6 x producer.
// ===========================================================================
template <int NC, int ST, int BN_ = 256>
struct GemmLnClusterCfg {
  static constexpr int BN = BN_;                        // columns per CTA (= d when NC = 1)
  static constexpr int TMEM_COLS = 2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512);   // two accumulators
  static constexpr int A_BYTES = 128 * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int XS = 2;                          // x chunk ring slots
  static constexpr int XCHUNK = 128 * 32 * 4;           // 128 rows x 32 fp32
  static constexpr int YCHUNK = 32 * 32 * 4;            // one warp's 32 rows x 32 fp32
  static constexpr int OFF_X = ST * STAGE;
  static constexpr int OFF_Y = OFF_X + XS * XCHUNK;
  static constexpr int OFF_BARS = OFF_Y + 4 * 2 * YCHUNK;
  static constexpr int STATS_BYTES = 2 * NC * 128 * 8;  // [slot][rank][row] (mean, M2)
  static constexpr int SMEM = OFF_BARS + 256 + STATS_BYTES + 1024;
  static constexpr int THREADS = 224;
  static_assert(SMEM <= 232448, "shared memory per CTA");
};

template <int NC, int ST, int BN_ = 256>
__global__ void __launch_bounds__(224, 1)
    gemm_ln_cluster_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                           const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_y,
                           EpiArgs ea, long long T, int K, DevStatus* status) {
  pdl_wait_then_release();
  using C = GemmLnClusterCfg<NC, ST, BN_>;
  constexpr int BN = C::BN;
  constexpr int XS = C::XS;
  constexpr int NCH = BN / 32;   // 32-column chunks per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::OFF_BARS);
  uint64_t* full = bars;                     // [ST]
  uint64_t* empty = bars + ST;               // [ST]
  uint64_t* acc_full = bars + 2 * ST;        // [2]
  uint64_t* acc_empty = bars + 2 * ST + 2;   // [2], one arrival per epilogue warp
  uint64_t* stats_full = bars + 2 * ST + 4;  // [2], one arrival per epilogue thread of each CTA of the cluster
  uint64_t* x_full = bars + 2 * ST + 6;      // [XS]
  uint64_t* x_empty = bars + 2 * ST + 8;     // [XS], one arrival per epilogue warp
  uint64_t* mma_done = bars + 2 * ST + 10;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * ST + 11);
  WaitCtl* wc = reinterpret_cast<WaitCtl*>(bars + 2 * ST + 12);   // 2 slots
  float2* stats = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(bars) + 256);
  uint8_t* xbuf = smem + C::OFF_X;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const long long MT = (T + 127) / 128;
  const long long cid = cluster_id_x(), ncl = cluster_count_x();
  const int n0 = (int)rank * BN;
  const int KT = (K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int i = 0; i < ST; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
      mbar_init(&stats_full[a], NC * 128);
    }
    for (int i = 0; i < XS; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 4);
    }
    mbar_init(mma_done, 1);
    waitctl_init(wc, status);
    fence_barrier_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_y);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  // Every CTA's barriers are initialised before any peer may arrive on them.
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---- producer: A / B k-tiles of every M tile of this cluster
      int last[ST];
      for (int i = 0; i < ST; ++i) last[i] = -1;
      long long it = 0;
      bool ok = true;
      for (long long mt = cid; mt < MT && ok; mt += ncl) {
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = (int)(it % ST);
          if (!mbar_wait(&empty[s], (uint32_t)((it / ST) & 1) ^ 1u, wc)) { ok = false; break; }
          if (it == 0 && cid == 0 && rank == 0 && wc->site == kSiteGemmOperand) continue;   // test hook
          mbar_arrive_expect_tx(&full[s], C::STAGE);
          uint8_t* st = smem + s * C::STAGE;
          tma_load_2d(st, &map_a, &full[s], kt * 64, (int)(mt * 128));
          tma_load_2d(st + C::A_BYTES, &map_b, &full[s], kt * 64, n0);
          last[s] = (int)(it / ST);
        }
      }
      for (int s = 0; s < ST; ++s)
        if (last[s] >= 0) mbar_drain(&full[s], last[s] & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer
      const uint32_t idesc = idesc_f16_f32(128, BN);
      long long it = 0;
      int ti = 0;
      bool ok = true;
      for (long long mt = cid; mt < MT && ok; mt += ncl, ++ti) {
        const int a = ti & 1;
        if (ti >= 2 && !mbar_wait(&acc_empty[a], ((ti >> 1) - 1) & 1, wc)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN;
        for (int kt = 0; kt < KT; ++kt, ++it) {
          const int s = (int)(it % ST);
          if (!mbar_wait(&full[s], (uint32_t)((it / ST) & 1), wc)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + s * C::STAGE);
          const uint32_t b_base = a_base + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_f16_ss(d_tmem, sdesc_kmajor(a_base + kk * 32, 128), sdesc_kmajor(b_base + kk * 32, 128), idesc,
                        (kt | kk) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[a]);
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp == 6) {
    if (lane == 0) {  // ---- x producer: the residual's 32-column chunks, tile after tile
      int last[XS];
      for (int i = 0; i < XS; ++i) last[i] = -1;
      long long g = 0;
      bool ok = true;
      for (long long mt = cid; mt < MT && ok; mt += ncl) {
        for (int cc = 0; cc < NCH; ++cc, ++g) {
          const int s = (int)(g % XS);
          if (!mbar_wait(&x_empty[s], (uint32_t)((g / XS) & 1) ^ 1u, wc)) { ok = false; break; }
          mbar_arrive_expect_tx(&x_full[s], C::XCHUNK);
          tma_load_2d(xbuf + s * C::XCHUNK, &map_x, &x_full[s], n0 + cc * 32, (int)(mt * 128));
          last[s] = (int)(g / XS);
        }
      }
      for (int s = 0; s < XS; ++s)
        if (last[s] >= 0) mbar_drain(&x_full[s], last[s] & 1);
    }
  } else {  // ---- epilogue warps 2..5, one output row per thread
    const int qd = warp & 3;
    const int row = qd * 32 + lane;
    const int d = ea.d;
    const float inv_d = 1.0f / (float)d;
    uint8_t* ystage = smem + C::OFF_Y + (warp - 2) * 2 * C::YCHUNK;
    // 16-byte piece c of row r of a 128B-swizzled box sits at r * 128 + 16 * (c ^ (r & 7)).
    const int xsw = row & 7, ysw = lane & 7;
    int ti = 0, nstore = 0;
    bool ok = true;
    for (long long mt = cid; mt < MT && ok; mt += ncl, ++ti) {
      const int a = ti & 1;
      const long long t = mt * 128 + row;
      const bool valid = t < T;
      // A padded query row's attention output (bias included) is zeroed:
      // y = LN2(x) there (BaselineSelfAttention, :121-122).
      const bool keep = ea.rowmask == nullptr || (valid && ea.rowmask[t] != 0);
      const uint32_t tl = tmem_base + a * BN + ((uint32_t)(qd * 32) << 16);
      if (!mbar_wait_warp(&acc_full[a], (uint32_t)(ti >> 1) & 1, wc)) break;
      tc_fence_after();
      // pass 1: r = x + (acc + b) back into TMEM, with the sums of (r - K) and
      // (r - K)^2 about the row's first value K here (a shift inside the
      // row's range keeps the one-pass variance free of cancellation).
      float s1 = 0.f, s2 = 0.f, shift = 0.f;
#pragma unroll 1
      for (int cc = 0; cc < NCH; ++cc) {
        const long long g = (long long)ti * NCH + cc;
        const int s = (int)(g % XS);
        if (!mbar_wait_warp(&x_full[s], (uint32_t)((g / XS) & 1), wc)) { ok = false; break; }
        uint32_t r[32];
        tmem_ld32(tl + cc * 32, r);
        const uint8_t* xr = xbuf + s * C::XCHUNK + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 xv = *reinterpret_cast<const float4*>(xr + ((c ^ xsw) << 4));
          const float4 bv = __ldg(reinterpret_cast<const float4*>(ea.bias + n0 + cc * 32) + c);
          const float a0 = xv.x + (keep ? __uint_as_float(r[4 * c + 0]) + bv.x : 0.f);
          const float a1 = xv.y + (keep ? __uint_as_float(r[4 * c + 1]) + bv.y : 0.f);
          const float a2 = xv.z + (keep ? __uint_as_float(r[4 * c + 2]) + bv.z : 0.f);
          const float a3 = xv.w + (keep ? __uint_as_float(r[4 * c + 3]) + bv.w : 0.f);
          if (cc == 0 && c == 0) shift = a0;
          const float d0 = a0 - shift, d1 = a1 - shift, d2 = a2 - shift, d3 = a3 - shift;
          s1 += (d0 + d1) + (d2 + d3);
          s2 += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
          r[4 * c + 0] = __float_as_uint(a0);
          r[4 * c + 1] = __float_as_uint(a1);
          r[4 * c + 2] = __float_as_uint(a2);
          r[4 * c + 3] = __float_as_uint(a3);
        }
        tmem_st32(tl + cc * 32, r);
        // The chunk's values were consumed (tmem_st32 waited for them) before
        // this release, so TMA may refill the slot.
        __syncwarp();
        if (lane == 0) mbar_arrive(&x_empty[s]);
      }
      if (!ok) break;
      const float dmean = s1 * (1.0f / (float)BN);
      const float mean_l = shift + dmean;
      const float m2 = fmaxf(s2 - s1 * dmean, 0.f);   // squared deviations about mean_l
      float mean = mean_l, M2 = m2;
      if constexpr (NC > 1) {
        // Exchange (mean, M2) of this row with every CTA of the cluster: store
        // the pair into each CTA's slot, then arrive (cluster-scope release of
        // that store) on each CTA's stats barrier, which expects one arrival
        // per epilogue thread of every CTA. Every wait stays bounded.
        const int slot = ti & 1;
        const uint32_t my_entry = smem_u32(&stats[(slot * NC + (int)rank) * 128 + row]);
        const uint32_t bar_local = smem_u32(&stats_full[slot]);
#pragma unroll 1
        for (int q = 0; q < NC; ++q) {
          st_cluster_v2(mapa_shared(my_entry, (uint32_t)q), mean_l, m2);
          mbar_arrive_cluster(mapa_shared(bar_local, (uint32_t)q));
        }
        if (!__all_sync(0xffffffffu, mbar_wait_cluster(&stats_full[slot], (uint32_t)(ti >> 1) & 1, wc))) break;
        mean = 0.f;
#pragma unroll
        for (int q = 0; q < NC; ++q) mean += stats[(slot * NC + q) * 128 + row].x;
        mean *= 1.0f / (float)NC;
        M2 = 0.f;
#pragma unroll
        for (int q = 0; q < NC; ++q) {
          const float2 e = stats[(slot * NC + q) * 128 + row];
          const float dm = e.x - mean;
          M2 += e.y + (float)BN * dm * dm;
        }
      }
      const float rstd = rsqrtf(M2 * inv_d + ea.eps);
      // pass 3: normalise this CTA's columns into the warp's staging buffers
      // and store each 32 x 32 box by TMA.
#pragma unroll 1
      for (int cc = 0; cc < NCH; ++cc, ++nstore) {
        uint32_t r[32];
        tmem_ld32(tl + cc * 32, r);
        uint8_t* yb = ystage + (nstore & 1) * C::YCHUNK;
        if (lane == 0) bulk_wait_read<1>();   // the store that last used this buffer has read it
        __syncwarp();
        uint8_t* yr = yb + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int col = n0 + cc * 32 + 4 * c;
          const float4 wv = __ldg(reinterpret_cast<const float4*>(ea.ln_w + col));
          const float4 bv = __ldg(reinterpret_cast<const float4*>(ea.ln_b + col));
          float4 o;
          o.x = (__uint_as_float(r[4 * c + 0]) - mean) * rstd * wv.x + bv.x;
          o.y = (__uint_as_float(r[4 * c + 1]) - mean) * rstd * wv.y + bv.y;
          o.z = (__uint_as_float(r[4 * c + 2]) - mean) * rstd * wv.z + bv.z;
          o.w = (__uint_as_float(r[4 * c + 3]) - mean) * rstd * wv.w + bv.w;
          *reinterpret_cast<float4*>(yr + ((c ^ ysw) << 4)) = o;
        }
        fence_proxy_async_smem();   // generic writes before the async-proxy (TMA) read
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_y, yb, n0 + cc * 32, (int)(mt * 128 + qd * 32));
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
    if (lane == 0) bulk_wait_all();   // this warp's y stores are complete
  }
  __syncthreads();
  if (threadIdx.x == 0 && waitctl_aborted(wc)) record_error(status, kErrTimeout, kGemmTma, 10 + NC);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
  // No CTA leaves while a peer may still write into its shared memory.
  cluster_sync_all();
}

}  // namespace b200l
