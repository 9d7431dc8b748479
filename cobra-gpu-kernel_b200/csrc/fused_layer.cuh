// fused_layer.cuh -- the whole layer in one persistent kernel for short
// sequences: y = LN2(x + Attn(LN1(x)) Wo^T + bo) with d_model in {64, 128},
// head_dim 32 and S <= 128 (the cfg1 / cfg2 benchmark shapes).
//
// One sequence (<= 128 tokens) fills the M = 128 rows of every tcgen05 tile,
// so h, q, k, v, the scores and ctx never leave the SM: per sequence the only
// HBM traffic is x in (read again for the residual, normally an L2 hit) and y
// out -- the layer's algorithmic 8*T*d bytes -- against 36*T*d for the
// three-kernel path. This is the B200 form of the reference's fused
// QKV+attention kernel (_qkvattn_kernel, torch_transformer_benchmark.py:654-741)
// carried through the out-projection and both LayerNorms.
//
// Two sequences are in flight, one per sequence slot (worker warpgroup), so
// the tensor core serves one while the other is in its LayerNorm / softmax /
// epilogue. Per sequence slot, TMEM (256 columns):
//   [0, 96)    q|k|v projection of one head (fp32); once read, q of the head
//              as fp16 pairs in [0, 16) (A operand of S = q k^T, from TMEM)
//   [96, 128)  O = P v of the head (fp32)
//   [128, 256) S = q k^T (fp32); P (fp16 pairs) overwrites [128, 192) in place;
//              after the last head, the out-projection accumulator [128, 128 + d)
// so the next sequence's first q|k|v projection can run during the LN2 epilogue.
// Shared memory per slot: A = LN1(x) fp16 (kept for every head's projection),
// C = ctx fp16 (A operand of the out-projection) as one [128 x 32] block of
// 64-byte rows per head, k [128 keys x 32] fp16 of the current head. v of
// head h is stored in ctx block h (token rows, 64-byte swizzle, the MN-major B
// operand of P v) and ctx of head h overwrites it once that P v completed.
// Weight tiles (q|k|v rows of one head, then Wo) stream from L2 through a
// 2-deep TMA ring shared by both slots.
// Per head the row warps run softmax(h), then the q|k|v epilogue of head h+1
// while P v of head h runs, then ctx(h): the P v and next-S round trips of the
// tensor core overlap row work instead of stalling it.
// Warps: 0 TMA producer, 1 / 2 MMA issuers of slot 0 / 1 (warp 1 owns TMEM;
// separate issuers keep one slot from stalling the other), 4-7 slot-0 rows, 8-11
// slot-1 rows (one token row per thread: q|k|v epilogue, softmax, ctx, LN2),
// 12-15 LayerNorm-1 of each slot's next sequence (warp per row, 16 rows of
// loads in flight), so x loads stay off the critical path. In the LN2
// epilogue each row warp loads its rows of the residual x and stores its rows
// of y by TMA (32-row x 32-column boxes through the k buffer and the ctx
// halves), so both move as full 128-byte lines; the warps of a slot meet only
// at the start of the next sequence (its k, v and ctx rows overlap other
// warps' x / y rows), and nothing ties the two slots together there.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace b200l {

struct FusedArgs {
  const float* x;
  float* y;
  const float* ln1_w;
  const float* ln1_b;
  const float* bqkv;
  const float* bo;
  const float* ln2_w;
  const float* ln2_b;
  float eps1, eps2;
  int B, S;
  int causal;
  float scale_log2;
  const uint8_t* mask;  // key-padding mask uint8 [B, S] (nonzero = valid), or nullptr
};

template <int DM>
struct FusedCfg {
  static constexpr int H = DM / 32;
  static constexpr int KC = DM / 64;                 // 128-byte atom columns along d
  static constexpr int WQ_BYTES = KC * 96 * 128;     // one head's q|k|v weight rows
  static constexpr int WO_BYTES = KC * DM * 128;     // Wo
  static constexpr int WBUF = ((WQ_BYTES > WO_BYTES ? WQ_BYTES : WO_BYTES) + 1023) / 1024 * 1024;
  static constexpr int A_BYTES = KC * 128 * 128;     // 128 token rows
  // k of the current head (128 keys x 32 fp16, 64-byte swizzle, 8 KB); the
  // buffer holds one 32-column fp32 chunk of x / y in the LN2 epilogue.
  static constexpr int KX_BYTES = 16384;
  static constexpr int SLOT = 2 * A_BYTES + KX_BYTES;
  static constexpr int PARAM_BYTES = 3 * DM * 4;     // bo, ln2_w, ln2_b in shared memory
  static constexpr int SMEM = 2 * WBUF + 2 * SLOT + 512 + PARAM_BYTES + 1024;
  static_assert(SMEM <= 232448, "fits the 227 KB opt-in shared memory of one CTA");
  static_assert(4 + 2 * 23 + 6 <= 64, "barrier block fits in 512 bytes");
};

// Per sequence slot; FB_XW + 3 q + i: row warp q's x chunk 0 (i = 0),
// chunks 1-2 (1) and chunk 3 (2).
enum FusedBar : int { FB_A_READY = 0, FB_A_FREE, FB_QKV_FULL, FB_QKV_FREE, FB_KQV_READY, FB_S_FULL, FB_P_READY,
                      FB_O_FULL, FB_CTX_READY, FB_OUT_FULL, FB_Y_READ, FB_XW, FB_COUNT = FB_XW + 12 };

template <int DM, bool KMASK>   // KMASK: a key-padding mask may be given
__global__ void __launch_bounds__(512, 1)
    fused_layer_kernel(const __grid_constant__ CUtensorMap map_wqkv, const __grid_constant__ CUtensorMap map_wo,
                       const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_y,
                       FusedArgs a, DevStatus* status) {
  using C = FusedCfg<DM>;
  constexpr int H = C::H;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sW = smem;
  uint8_t* sSlot = smem + 2 * C::WBUF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sSlot + 2 * C::SLOT);
  uint64_t* w_full = bars;
  uint64_t* w_empty = bars + 2;
  uint64_t* mma_done = bars + 4 + 2 * FB_COUNT;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  WaitCtl* wc = reinterpret_cast<WaitCtl*>(mma_done + 4);   // slots 4-5 past mma_done
  // bo | ln2_w | ln2_b, read by every row thread in the out-projection epilogue.
  float* sprm = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 512);
  auto sb = [&](int s, int i) { return bars + 4 + FB_COUNT * s + i; };
  auto slot_a = [&](int s) { return sSlot + s * C::SLOT; };
  auto slot_c = [&](int s) { return sSlot + s * C::SLOT + C::A_BYTES; };
  auto slot_k = [&](int s) { return sSlot + s * C::SLOT + 2 * C::A_BYTES; };

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int npairs = (a.B + 1) / 2;
  const int S = a.S;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 2);   // released by both slots' MMA threads
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(sb(s, FB_A_READY), 2);
      mbar_init(sb(s, FB_A_FREE), 1);
      mbar_init(sb(s, FB_QKV_FULL), 1);
      mbar_init(sb(s, FB_QKV_FREE), 4);
      mbar_init(sb(s, FB_KQV_READY), 4);
      mbar_init(sb(s, FB_S_FULL), 1);
      mbar_init(sb(s, FB_P_READY), 4);
      mbar_init(sb(s, FB_O_FULL), 1);
      mbar_init(sb(s, FB_CTX_READY), 4);
      mbar_init(sb(s, FB_OUT_FULL), 1);
      mbar_init(sb(s, FB_Y_READ), 4);     // every row warp's y stores have read the chunk buffers
      for (int i = 0; i < 12; ++i) mbar_init(sb(s, FB_XW + i), 1);
    }
    mbar_init(mma_done, 2);
    waitctl_init(wc, status);
    fence_barrier_init();
    tma_prefetch_desc(&map_wqkv);
    tma_prefetch_desc(&map_wo);
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_y);
  }
  for (int i = threadIdx.x; i < DM; i += blockDim.x) {
    sprm[i] = a.bo[i];
    sprm[DM + i] = a.ln2_w[i];
    sprm[2 * DM + i] = a.ln2_b[i];
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // x is read twice (LN1, then the residual about two sequence pairs later):
  // LN1's loads keep it in L2 (evict_last), the residual's TMA read and y's
  // TMA store mark their lines evict_first, so the second read of x hits L2.
  const uint64_t pol_keep = l2_policy_evict_last(), pol_once = l2_policy_evict_first();

  if (warp == 0) {
    if (lane == 0) {  // ======================= TMA producer: weight tiles
      int wt = 0, last[2] = {-1, -1};
      bool ok = true;
      for (int pair = blockIdx.x; pair < npairs && ok; pair += gridDim.x) {
        for (int t = 0; t <= H; ++t, ++wt) {
          const int b = wt & 1;
          if (!mbar_wait(&w_empty[b], ((wt >> 1) & 1) ^ 1, wc)) { ok = false; break; }
          uint8_t* dst = sW + b * C::WBUF;
          if (t < H) {
            mbar_arrive_expect_tx(&w_full[b], C::WQ_BYTES);
            for (int kc = 0; kc < C::KC; ++kc)
              for (int part = 0; part < 3; ++part)
                tma_load_2d(dst + kc * (96 * 128) + part * (32 * 128), &map_wqkv, &w_full[b], kc * 64,
                            part * DM + t * 32);
          } else {
            mbar_arrive_expect_tx(&w_full[b], C::WO_BYTES);
            for (int kc = 0; kc < C::KC; ++kc)
              tma_load_2d(dst + kc * (DM * 128), &map_wo, &w_full[b], kc * 64, 0);
          }
          last[b] = wt;
        }
      }
      for (int b = 0; b < 2; ++b)
        if (last[b] >= 0) mbar_drain(&w_full[b], (last[b] >> 1) & 1);
    }
  } else if (warp == 1 || warp == 2) {
    if (lane == 0) {  // ======================= MMA issuer of slot (warp - 1)
      const int s = warp - 1;
      const uint32_t id_qkv = idesc_f16_f32(128, 96);
      const uint32_t id_s = idesc_f16_f32(128, 128);
      const uint32_t id_o = idesc_f16_f32(128, 32);
      const uint32_t id_out = idesc_f16_f32(128, DM);
      const uint32_t t_slot = tmem_base + s * 256;
      const uint32_t abase = smem_u32(slot_a(s));
      const uint32_t cbase = smem_u32(slot_c(s));
      const uint32_t kbase = smem_u32(slot_k(s));
      int wt = 0, pi = 0;
      bool ok = true;
      // q|k|v projection of head h from weight tile wt; both slots' issuers
      // read the same tile and each releases it once its MMAs finish.
      auto issue_qkv = [&](int h, bool active) -> bool {
        const int b = wt & 1;
        const int n = pi * H + h;
        if (!mbar_wait(&w_full[b], (wt >> 1) & 1, wc)) return false;
        if (active) {
          if (n > 0 && !mbar_wait(sb(s, FB_QKV_FREE), (n - 1) & 1, wc)) return false;
          tc_fence_after();
          const uint32_t wbase = smem_u32(sW + b * C::WBUF);
#pragma unroll
          for (int k = 0; k < DM / 16; ++k) {
            const uint32_t oa = (uint32_t)(k >> 2) * 16384 + (k & 3) * 32;
            const uint32_t ow = (uint32_t)(k >> 2) * (96 * 128) + (k & 3) * 32;
            umma_f16_ss(t_slot, sdesc_kmajor(abase + oa, 128), sdesc_kmajor(wbase + ow, 128), id_qkv,
                        k > 0 ? 1u : 0u);
          }
          umma_commit(sb(s, FB_QKV_FULL));
          // The last projection of the sequence is the last reader of A: LN1
          // may refill it as soon as that MMA completes.
          if (h == H - 1) umma_commit(sb(s, FB_A_FREE));
        }
        umma_commit(&w_empty[b]);
        ++wt;
        return true;
      };
      for (int pair = blockIdx.x; pair < npairs && ok; pair += gridDim.x, ++pi) {
        // slot 1 may be empty in the last pair: it still walks the weight ring
        const bool active = 2 * pair + s < a.B;
        if (active && !mbar_wait(sb(s, FB_A_READY), pi & 1, wc)) { ok = false; break; }
        if (!issue_qkv(0, active)) { ok = false; break; }
        for (int h = 0; h < H && ok; ++h) {
          const int n = pi * H + h;
          if (active) {  // S = q k^T, q (fp16) from TMEM [0, 16)
            // S overwrites P of the previous head: its P v completed (waited below).
            if (!mbar_wait(sb(s, FB_KQV_READY), n & 1, wc)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 2; ++k)
              umma_f16_ts(t_slot + 128, t_slot + k * 8, sdesc_kmajor(kbase + k * 32, 64), id_s, k > 0 ? 1u : 0u);
            umma_commit(sb(s, FB_S_FULL));
          }
          // The next head's projection runs while this head's softmax does; it
          // overwrites q in [0, 16), so it waits for this S to complete.
          if (h + 1 < H) {
            if (active && !mbar_wait(sb(s, FB_S_FULL), n & 1, wc)) { ok = false; break; }
            if (!issue_qkv(h + 1, active)) { ok = false; break; }
          }
          if (active) {  // O = P v, P from TMEM
            if (!mbar_wait(sb(s, FB_P_READY), n & 1, wc)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < 8; ++k)
              // B = v [16 keys x 32] in ctx block h, rows of 64 B from key 16k:
              // MN-major, one 32-column swizzle atom along N, 8-key row groups
              // 512 B apart.
              umma_f16_ts(t_slot + 96, t_slot + 128 + k * 8,
                          sdesc_kmajor(cbase + (uint32_t)h * 8192 + (uint32_t)k * 1024, 64), id_o | (1u << 16),
                          k > 0 ? 1u : 0u);
            umma_commit(sb(s, FB_O_FULL));
            // The next S (or the out-projection) overwrites P: wait for this P v.
            if (!mbar_wait(sb(s, FB_O_FULL), n & 1, wc)) { ok = false; break; }
          }
        }
        if (!ok) break;
        {  // out-projection: ctx Wo^T
          const int b = wt & 1;
          if (!mbar_wait(&w_full[b], (wt >> 1) & 1, wc)) { ok = false; break; }
          if (active) {
            if (!mbar_wait(sb(s, FB_CTX_READY), pi & 1, wc)) { ok = false; break; }
            tc_fence_after();
            const uint32_t wbase = smem_u32(sW + b * C::WBUF);
#pragma unroll
            for (int k = 0; k < DM / 16; ++k) {
              // ctx: one [128 x 32] fp16 block per head, 64-byte rows
              const uint32_t oc = (uint32_t)(k >> 1) * 8192 + (k & 1) * 32;
              const uint32_t ow = (uint32_t)(k >> 2) * (DM * 128) + (k & 3) * 32;
              umma_f16_ss(t_slot + 128, sdesc_kmajor(cbase + oc, 64), sdesc_kmajor(wbase + ow, 128), id_out,
                          k > 0 ? 1u : 0u);
            }
            umma_commit(sb(s, FB_OUT_FULL));
          }
          umma_commit(&w_empty[b]);
          ++wt;
        }
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp >= 12) {  // ======================= LN1: warps 12,13 -> slot 0; 14,15 -> slot 1
    const int s = (warp - 12) >> 1;
    const int rbeg = ((warp - 12) & 1) * 64;
    const uint32_t a_base = smem_u32(slot_a(s));
    const float inv_d = 1.0f / (float)DM;
    // Eight lanes per row, four rows per warp instruction: lane (grp, l) holds
    // columns 32*m + 4*l (m < NV) of row 4*i + grp, so every load instruction
    // reads four 128-byte segments and a row reduces in three shuffle steps.
    constexpr int NV = DM / 32;               // float4 per lane per row
    const int grp = lane >> 3, l8 = lane & 7;
    float4 w4[NV], b4[NV];
#pragma unroll
    for (int m = 0; m < NV; ++m) {
      w4[m] = __ldg(reinterpret_cast<const float4*>(a.ln1_w + 32 * m + 4 * l8));
      b4[m] = __ldg(reinterpret_cast<const float4*>(a.ln1_b + 32 * m + 4 * l8));
    }
    int pi = 0;
    for (int pair = blockIdx.x; pair < npairs; pair += gridDim.x, ++pi) {
      const int seq = 2 * pair + s;
      if (seq >= a.B) break;
      const long long t0 = (long long)seq * S;
      {  // pull this slot's next sequence (these 64 rows) toward L2
        const int nseq = seq + 2 * (int)gridDim.x;
        if (nseq < a.B && rbeg < S) {
          const int rows = min(64, S - rbeg);
          const char* p = reinterpret_cast<const char*>(a.x + ((long long)nseq * S + rbeg) * DM);
          const int lines = (rows * DM * 4 + 127) / 128;
          for (int i = lane; i < lines; i += 32) prefetch_l2(p + (long long)i * 128);
        }
      }
      // A of this slot is free once the previous sequence's last projection was read.
      if (!mbar_wait(sb(s, FB_A_FREE), (pi & 1) ^ 1, wc)) break;
      constexpr int IT = 2;   // row groups per batch: 8 rows, 2*NV loads in flight per lane
#pragma unroll 1
      for (int r0 = rbeg; r0 < rbeg + 64; r0 += 4 * IT) {
        float4 v[IT][NV];
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          const int r = r0 + 4 * it + grp;
#pragma unroll
          for (int m = 0; m < NV; ++m)
            v[it][m] = (r < S) ? ldg_stream_f4_hint(a.x + (t0 + r) * DM + 32 * m + 4 * l8, pol_keep)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        float red[IT], mean[IT], rstd[IT];
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          float sm = 0.f;
#pragma unroll
          for (int m = 0; m < NV; ++m) sm += (v[it][m].x + v[it][m].y) + (v[it][m].z + v[it][m].w);
          red[it] = sm;
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1)
#pragma unroll
          for (int it = 0; it < IT; ++it) red[it] += __shfl_xor_sync(0xffffffffu, red[it], o);
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          mean[it] = red[it] * inv_d;
          float sq = 0.f;
#pragma unroll
          for (int m = 0; m < NV; ++m) {
            v[it][m].x -= mean[it]; v[it][m].y -= mean[it]; v[it][m].z -= mean[it]; v[it][m].w -= mean[it];
            sq += (v[it][m].x * v[it][m].x + v[it][m].y * v[it][m].y) + (v[it][m].z * v[it][m].z + v[it][m].w * v[it][m].w);
          }
          red[it] = sq;
        }
#pragma unroll
        for (int o = 1; o < 8; o <<= 1)
#pragma unroll
          for (int it = 0; it < IT; ++it) red[it] += __shfl_xor_sync(0xffffffffu, red[it], o);
#pragma unroll
        for (int it = 0; it < IT; ++it) {
          rstd[it] = rsqrtf(red[it] * inv_d + a.eps1);
          const int r = r0 + 4 * it + grp;
#pragma unroll
          for (int m = 0; m < NV; ++m) {
            const int k = 32 * m + 4 * l8;
            uint32_t lo = 0, hi = 0;
            if (r < S) {
              lo = pack_half2(v[it][m].x * rstd[it] * w4[m].x + b4[m].x, v[it][m].y * rstd[it] * w4[m].y + b4[m].y);
              hi = pack_half2(v[it][m].z * rstd[it] * w4[m].z + b4[m].z, v[it][m].w * rstd[it] * w4[m].w + b4[m].w);
            }
            st_shared_v2(a_base + (k >> 6) * 16384 + swz_offset(r, (k & 63) >> 3, 128) + (k & 7) * 2, lo, hi);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(sb(s, FB_A_READY));
    }
  } else if (warp >= 4) {  // ======================= row workers (warps 4-11), one token per thread
    const int s = (warp - 4) >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tb = tmem_base + (uint32_t)(s * 256) + ((uint32_t)(q * 32) << 16);
    const uint32_t c_base = smem_u32(slot_c(s));
    const uint32_t k_base = smem_u32(slot_k(s));
    const float sl2 = a.scale_log2;
    const float inv_d = 1.0f / (float)DM;
    int pi = 0;
    constexpr int NXC = DM / 32;   // 32-column fp32 chunks of x / y per row: 4 (d=128) or 2 (d=64)
    for (int pair = blockIdx.x; pair < npairs; pair += gridDim.x, ++pi) {
      const int seq = 2 * pair + s;
      if (seq >= a.B) break;
      const long long t0 = (long long)seq * S;
      // k, v and ctx rows (64 bytes) overlap other warps' rows of the x / y
      // chunks (128 bytes): every row warp's y stores of the previous
      // sequence must have read the buffers before this sequence writes them.
      if (pi > 0) {
        if (lane == 0) {
          bulk_wait_read_all();
          mbar_arrive(sb(s, FB_Y_READ));
        }
        if (!mbar_wait_warp(sb(s, FB_Y_READ), (pi - 1) & 1, wc)) break;
      }
      // Keys this row may see, one bit each: valid (mask), inside S, causal.
      // A padded query row (mask byte 0) keeps y = LN2(x): its attention
      // output, bias included, is zeroed (BaselineSelfAttention :106-109, :121-122).
      const int lim = a.causal ? min(S, row + 1) : S;  // keys [0, lim) are in range
      uint32_t vb[4] = {0u, 0u, 0u, 0u};
      bool qkeep = true;
      if constexpr (KMASK) {
        uint32_t kb[4] = {0xffffffffu, 0xffffffffu, 0xffffffffu, 0xffffffffu};
        if (a.mask != nullptr) {
          key_mask_load<4>(a.mask + t0, 0, S, lane, kb);
          key_mask_ballot<4>(kb);
          const uint32_t mine = q == 0 ? kb[0] : q == 1 ? kb[1] : q == 2 ? kb[2] : kb[3];
          qkeep = ((mine >> lane) & 1u) != 0u;
        }
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const int nb = lim - 32 * w;
          vb[w] = kb[w] & (nb >= 32 ? 0xffffffffu : (nb <= 0 ? 0u : ((1u << nb) - 1u)));
        }
      }
      const bool full = KMASK ? (vb[0] & vb[1] & vb[2] & vb[3]) == 0xffffffffu : (lim == 128);
      // q|k|v epilogue of head h: bias, fp16; q -> TMEM [0, 16) (the A operand
      // of S), k -> the k buffer, v -> ctx block h (read by P v of head h
      // before ctx of head h is written there).
      auto qkv_epilogue = [&](int h) -> bool {
        const int n = pi * H + h;
        if (!mbar_wait_warp(sb(s, FB_QKV_FULL), n & 1, wc)) return false;
        tc_fence_after();
        uint32_t r[32], pk[16];
        tmem_ld32(tb + 0, r);
        const float4* bq = reinterpret_cast<const float4*>(a.bqkv + 32 * h);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 bb = __ldg(bq + i);
          const float2 v01 = __fadd2_rn(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])),
                                        make_float2(bb.x, bb.y));
          const float2 v23 = __fadd2_rn(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])),
                                        make_float2(bb.z, bb.w));
          pk[2 * i] = pack_half2(v01.x, v01.y);
          pk[2 * i + 1] = pack_half2(v23.x, v23.y);
        }
        tmem_st16(tb + 0, pk);
        // k, then v: token rows of 64 bytes, 64-byte swizzle
        auto kv_row = [&](int part, uint32_t dst) {
          tmem_ld32(tb + 32 * part, r);
          const float4* bb4 = reinterpret_cast<const float4*>(a.bqkv + part * DM + 32 * h);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(bb4 + i);
            const float2 v01 = __fadd2_rn(make_float2(__uint_as_float(r[4 * i]), __uint_as_float(r[4 * i + 1])),
                                          make_float2(bb.x, bb.y));
            const float2 v23 = __fadd2_rn(make_float2(__uint_as_float(r[4 * i + 2]), __uint_as_float(r[4 * i + 3])),
                                          make_float2(bb.z, bb.w));
            pk[2 * i] = pack_half2(v01.x, v01.y);
            pk[2 * i + 1] = pack_half2(v23.x, v23.y);
          }
#pragma unroll
          for (int c = 0; c < 4; ++c)
            st_shared_v4(dst + row * 64 + ((c ^ ((row >> 1) & 3)) << 4), pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                         pk[4 * c + 3]);
        };
        kv_row(1, k_base);
        kv_row(2, c_base + (uint32_t)h * 8192);
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(sb(s, FB_QKV_FREE));   // q|k|v accumulator [0, 96) read
          mbar_arrive(sb(s, FB_KQV_READY));
        }
        return true;
      };
      bool ok = qkv_epilogue(0);
      for (int h = 0; h < H && ok; ++h) {
        const int n = pi * H + h;
        // ---- softmax of S = q k^T (one row per thread, exact: S <= 128 keys)
        if (!mbar_wait_warp(sb(s, FB_S_FULL), n & 1, wc)) { ok = false; break; }
        tc_fence_after();
        float m8[8];   // eight independent running maxima: short dependency chains
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = -INFINITY;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tb + 128 + 32 * c, r);
          const uint32_t vw = !KMASK ? 0u : c == 0 ? vb[0] : c == 1 ? vb[1] : c == 2 ? vb[2] : vb[3];
          if (full) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              m8[i & 7] = fmax3f(m8[i & 7], __uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              m8[i & 7] = fmaxf(m8[i & 7], (KMASK ? ((vw >> i) & 1u) != 0u : 32 * c + i < lim)
                                                 ? __uint_as_float(r[i]) : -INFINITY);
          }
        }
        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                               fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        const float ms = (mx == -INFINITY) ? 0.f : mx * sl2;   // every key masked: p = 0, l = 0
        const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-ms, -ms);
        float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32], pk[16];
          tmem_ld32(tb + 128 + 32 * c, r);
          const uint32_t vw = !KMASK ? 0u : c == 0 ? vb[0] : c == 1 ? vb[1] : c == 2 ? vb[2] : vb[3];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            // masked keys: exp2(-inf) = 0
            const int k0 = 32 * c + 2 * i;
            const bool v0 = KMASK ? ((vw >> (2 * i)) & 1u) != 0u : k0 < lim;
            const bool v1 = KMASK ? ((vw >> (2 * i + 1)) & 1u) != 0u : k0 + 1 < lim;
            const float s0 = (full || v0) ? __uint_as_float(r[2 * i]) : -INFINITY;
            const float s1 = (full || v1) ? __uint_as_float(r[2 * i + 1]) : -INFINITY;
            const float2 xx = __ffma2_rn(make_float2(s0, s1), sc2, nm2);
            const float2 pp = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
            acc[i & 1] = __fadd2_rn(acc[i & 1], pp);
            pk[i] = pack_half2(pp.x, pp.y);
          }
          tmem_st16(tb + 128 + 16 * c, pk);  // P overwrites the S columns already read
        }
        const float2 a01 = __fadd2_rn(acc[0], acc[1]);
        const float l = a01.x + a01.y;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(sb(s, FB_P_READY));
        // ---- the next head's q|k|v epilogue while this head's P v runs
        if (h + 1 < H && !qkv_epilogue(h + 1)) { ok = false; break; }
        // ---- ctx columns of head h = O / l, fp16, into ctx block h (over v of head h)
        if (!mbar_wait_warp(sb(s, FB_O_FULL), n & 1, wc)) { ok = false; break; }
        tc_fence_after();
        {
          uint32_t r[32];
          tmem_ld32(tb + 96, r);
          const float il = l > 0.f ? 1.0f / l : 0.f;
          const float2 il2 = make_float2(il, il);
          const uint32_t cb = c_base + (uint32_t)h * 8192 + row * 64;
#pragma unroll
          for (int c = 0; c < 4; ++c)
            st_shared_v4(cb + ((c ^ ((row >> 1) & 3)) << 4),
                         pack_f2h(__fmul2_rn(make_float2(__uint_as_float(r[8 * c + 0]), __uint_as_float(r[8 * c + 1])), il2)),
                         pack_f2h(__fmul2_rn(make_float2(__uint_as_float(r[8 * c + 2]), __uint_as_float(r[8 * c + 3])), il2)),
                         pack_f2h(__fmul2_rn(make_float2(__uint_as_float(r[8 * c + 4]), __uint_as_float(r[8 * c + 5])), il2)),
                         pack_f2h(__fmul2_rn(make_float2(__uint_as_float(r[8 * c + 6]), __uint_as_float(r[8 * c + 7])), il2)));
        }
      }
      if (!ok) break;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(sb(s, FB_CTX_READY));
      // ---- out-projection epilogue: r = x + (acc + bo), LN2, y.
      // Each row warp moves its own 32 rows: lane 0 loads x and stores y as
      // 32-row x 32-column fp32 TMA boxes (4 KB, 128-byte swizzle) through
      // three 16 KB chunk buffers of the slot -- chunk 0, then chunk 3, through
      // the k buffer (free since the last S), chunks 1-2 through the two halves
      // of ctx once the out-projection has read it. Within the epilogue every
      // buffer is used row by row, so no barrier couples the warps here, nor
      // the two slots.
      uint8_t* kxp = slot_k(s);
      uint8_t* cxp = slot_c(s);
      auto xchunk = [&](int cc) -> uint8_t* { return (cc == 0 || cc == 3) ? kxp : cxp + (cc - 1) * 16384; };
      uint64_t* xbar = sb(s, FB_XW + 3 * q);   // this warp's x chunk 0 | chunks 1-2 | chunk 3
      auto x_load = [&](int cc, uint64_t* bar) {
        tma_load_3d_hint(xchunk(cc) + q * 4096, &map_x, bar, cc * 32, q * 32, seq, pol_once);
      };
      auto y_store = [&](int cc) { tma_store_3d_hint(&map_y, xchunk(cc) + q * 4096, cc * 32, q * 32, seq, pol_once); };
      if (lane == 0) {
        mbar_arrive_expect_tx(&xbar[0], 4096);
        x_load(0, &xbar[0]);
      }
      if (!mbar_wait_warp(sb(s, FB_OUT_FULL), pi & 1, wc)) break;
      tc_fence_after();
      if (lane == 0) {
        mbar_arrive_expect_tx(&xbar[1], NXC > 2 ? 8192 : 4096);
        x_load(1, &xbar[1]);
        if constexpr (NXC > 2) x_load(2, &xbar[1]);
      }
      {
        // Statistics in one pass over the shifted values r - r0 (r0 = the row's
        // first element): var = E[(r-r0)^2] - E[r-r0]^2 has no cancellation when
        // the row's spread is small next to its mean.
        float shift = 0.f;
        float2 sum2 = make_float2(0.f, 0.f), sq2 = make_float2(0.f, 0.f);   // packed fp32x2 partials
        // Chunks cc0 .. cc0 + NCH - 1 from one TMEM round trip; r = x + (acc +
        // bo) goes back to TMEM for the second pass. NCH is 1, or 2 where
        // registers allow (the masked variant keeps 1).
        auto stats = [&](auto nch, int cc0) {
          constexpr int NCH = decltype(nch)::value;
          uint32_t r[32 * NCH];
          if constexpr (NCH == 2) tmem_ld64(tb + 128 + 32 * cc0, r);
          else tmem_ld32(tb + 128 + 32 * cc0, r);
#pragma unroll
          for (int HH = 0; HH < NCH; ++HH) {
            const int cc = cc0 + HH;
            const uint8_t* src = xchunk(cc);
#pragma unroll
            for (int c = 0; c < 8; ++c) {
              const int col = cc * 32 + 4 * c;
              const float4 x4 = *reinterpret_cast<const float4*>(src + row * 128 + ((c ^ (row & 7)) << 4));
              const float4 bb = *reinterpret_cast<const float4*>(sprm + col);
              const int i0 = 32 * HH + 4 * c;
              // r = x + (acc + bo), in pairs; a padded row keeps r = x.
              const float2 acc01 = make_float2(__uint_as_float(r[i0 + 0]), __uint_as_float(r[i0 + 1]));
              const float2 acc23 = make_float2(__uint_as_float(r[i0 + 2]), __uint_as_float(r[i0 + 3]));
              float2 a01 = make_float2(x4.x, x4.y), a23 = make_float2(x4.z, x4.w);
              const float2 o01 = __fadd2_rn(acc01, make_float2(bb.x, bb.y));
              const float2 o23 = __fadd2_rn(acc23, make_float2(bb.z, bb.w));
              a01 = qkeep ? __fadd2_rn(a01, o01) : a01;
              a23 = qkeep ? __fadd2_rn(a23, o23) : a23;
              if (cc == 0 && c == 0) shift = a01.x;
              const float2 nsh = make_float2(-shift, -shift);
              const float2 d01 = __fadd2_rn(a01, nsh), d23 = __fadd2_rn(a23, nsh);
              sum2 = __fadd2_rn(sum2, __fadd2_rn(d01, d23));
              sq2 = __ffma2_rn(d01, d01, sq2);
              sq2 = __ffma2_rn(d23, d23, sq2);
              r[i0 + 0] = __float_as_uint(a01.x);
              r[i0 + 1] = __float_as_uint(a01.y);
              r[i0 + 2] = __float_as_uint(a23.x);
              r[i0 + 3] = __float_as_uint(a23.y);
            }
          }
          if constexpr (NCH == 2) tmem_st64(tb + 128 + 32 * cc0, r);
          else tmem_st32(tb + 128 + 32 * cc0, r);
        };
        using One = std::integral_constant<int, 1>;
        using Two = std::integral_constant<int, KMASK ? 1 : 2>;
        if (!mbar_wait_warp(&xbar[0], pi & 1, wc)) break;
        stats(One{}, 0);
        if constexpr (NXC > 2) {   // chunk 0 consumed: chunk 3 into the k buffer
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            mbar_arrive_expect_tx(&xbar[2], 4096);
            x_load(3, &xbar[2]);
          }
        }
        if (!mbar_wait_warp(&xbar[1], pi & 1, wc)) break;
        if constexpr (NXC > 2) {
          stats(Two{}, 1);
          if constexpr (KMASK) stats(One{}, 2);
          if (!mbar_wait_warp(&xbar[2], pi & 1, wc)) break;
          stats(One{}, 3);
        } else {
          stats(One{}, 1);
        }
        const float dmean = (sum2.x + sum2.y) * inv_d;
        const float mean = shift + dmean;
        const float rstd = rsqrtf(fmaxf((sq2.x + sq2.y) * inv_d - dmean * dmean, 0.f) + a.eps2);
        // y = (r - mean) * rstd * w + b as (r * rstd - mean * rstd) * w + b, in pairs.
        const float2 rs2 = make_float2(rstd, rstd), nm2 = make_float2(-mean * rstd, -mean * rstd);
        // Second pass: y from r (kept in TMEM by the first pass), staged over
        // this row's x chunk in place and stored by the warp's lane 0 (rows
        // past S are clipped).
        auto y_chunk = [&](const uint32_t (&r)[32], int cc) {
          const uint32_t dst = smem_u32(xchunk(cc)) + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const int col = cc * 32 + 4 * c;
            const float4 wv = *reinterpret_cast<const float4*>(sprm + DM + col);
            const float4 bb = *reinterpret_cast<const float4*>(sprm + 2 * DM + col);
            const float2 t01 = __ffma2_rn(make_float2(__uint_as_float(r[4 * c + 0]), __uint_as_float(r[4 * c + 1])), rs2, nm2);
            const float2 t23 = __ffma2_rn(make_float2(__uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3])), rs2, nm2);
            const float2 y01 = __ffma2_rn(t01, make_float2(wv.x, wv.y), make_float2(bb.x, bb.y));
            const float2 y23 = __ffma2_rn(t23, make_float2(wv.z, wv.w), make_float2(bb.z, bb.w));
            st_shared_v4(dst + ((c ^ (row & 7)) << 4), __float_as_uint(y01.x), __float_as_uint(y01.y),
                         __float_as_uint(y23.x), __float_as_uint(y23.y));
          }
        };
        // One TMEM round trip per chunk (a 64-column r spills here). Bulk
        // groups: [y0], [y1 y2], then y3 over y0 in the k buffer once the
        // first group has read it.
        uint32_t r[32];
#pragma unroll 1
        for (int cc = 0; cc < NXC; ++cc) {
          if (cc == 3) {
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
          }
          tmem_ld32(tb + 128 + 32 * cc, r);
          y_chunk(r, cc);
          fence_proxy_async_smem();   // generic writes before the async-proxy (TMA) reads
          __syncwarp();
          if (lane == 0) {
            y_store(cc);
            if (cc != 1 || NXC == 2) bulk_commit();
          }
        }
      }
      tc_fence_before();   // TMEM reads of this sequence done before the next S MMA
    }
  }
  if (warp >= 4 && warp < 12) {   // row warps: their y stores complete before exit
    if (lane == 0) bulk_wait_all();
  }
  __syncthreads();
  if (threadIdx.x == 0 && waitctl_aborted(wc)) record_error(status, kErrTimeout, kFusedLayer, 0);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace b200l
