// attn.cuh -- K2: flash attention on tcgen05 (scores never leave the SM).
//
// ctx[b, s, h*dh + j] = sum_k softmax_k(q.k / sqrt(dh)) v[k, j] per (b, h),
// restating BaselineSelfAttention.forward (torch_transformer_benchmark.py:98,
// :100-104 causal mask, :112-113 fp32 softmax then probs @ v) without
// materialising [B,H,S,S]; the reference's fused counterpart is _attn_kernel
// (:572-649).
//
// Persistent CTAs walk work items (b, h, 128-query tile). Per item:
//   S = Q K_j^T       tcgen05, M=128 queries x N=BN keys, K=dhp, fp32 in TMEM
//   softmax           one thread per query row: the row's BN scores come from
//                     TMEM into registers, max / exp2 / sum are thread-local
//                     (no shuffles), P is written as fp16 to shared memory in
//                     the swizzled K-major operand layout
//   O += P V_j        tcgen05, M=128 x N=dhp, K=BN, fp32 O stays in TMEM
// The running max is updated lazily: O and l are rescaled only when the row
// max grows by more than 2^8 (log2 domain), so p <= 256 and fp16 P is safe.
// Roles: warp 0 TMA producer (Q double-buffered across items, K/V 2 stages),
// warp 1 MMA issuer + TMEM owner, warps 2-5 softmax / correction / epilogue.
// The S buffer is released as soon as a row is in registers, so the MMA of
// tile j+1 overlaps the exponentials of tile j.
#pragma once

#include "common.cuh"

namespace b200l {

struct AttnArgs {
  __half* ctx;  // [B*S, d]
  int B, S, H, dh, d;
  int causal;
  float scale_log2;  // dh^-0.5 * log2(e)
  int num_items;     // B*H*ceil(S/128)
  const uint8_t* kmask;  // key-padding mask uint8 [B, S] (nonzero = valid), or nullptr
};

template <int DHP, int BN>
struct AttnCfg {
  static constexpr int QKROW = DHP >= 64 ? 128 : 64;        // bytes per swizzled row of Q/K tiles
  static constexpr int QKC = DHP * 2 / QKROW;               // atom columns along dh
  static constexpr int Q_BYTES = 128 * DHP * 2;
  static constexpr int K_BYTES = BN * DHP * 2;
  static constexpr int V_BYTES = DHP * BN * 2;              // v^T tile: DHP rows x BN keys
  static constexpr int P_BYTES = 128 * BN * 2;
  static constexpr int QST = (2 * Q_BYTES + 2 * (K_BYTES + V_BYTES) + P_BYTES <= 200 * 1024) ? 2 : 1;
  static constexpr int KVST = 2;
  static constexpr int SMEM = QST * Q_BYTES + KVST * (K_BYTES + V_BYTES) + P_BYTES + 256 + 1024;
  static constexpr int S_COL = 0;
  static constexpr int O_COL = BN;
  static constexpr int TMEM_COLS = (BN + DHP) <= 256 ? 256 : 512;
};

template <int DHP, int BN, bool KMASK>   // KMASK: a key-padding mask may be given
__global__ void __launch_bounds__(192, 1)
    attn_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                const __grid_constant__ CUtensorMap map_vt, AttnArgs args, DevStatus* status) {
  pdl_wait_then_release();
  using C = AttnCfg<DHP, BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::QST * C::Q_BYTES;
  uint8_t* sV = sK + C::KVST * C::K_BYTES;
  uint8_t* sP = sV + C::KVST * C::V_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::P_BYTES);
  uint64_t* q_full = bars;        // [2]
  uint64_t* q_empty = bars + 2;   // [2]
  uint64_t* kv_full = bars + 4;   // [2]
  uint64_t* kv_empty = bars + 6;  // [2]
  uint64_t* s_full = bars + 8;
  uint64_t* s_free = bars + 9;
  uint64_t* p_full = bars + 10;
  uint64_t* pv_done = bars + 11;
  uint64_t* mma_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  WaitCtl* wc = reinterpret_cast<WaitCtl*>(bars + 14);   // bars 14-15

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = args.S;
  const int QT = (S + 127) / 128;
  const int NKV_ALL = (S + BN - 1) / BN;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    mbar_init(pv_done, 1);
    mbar_init(mma_done, 1);
    waitctl_init(wc, status);
    fence_barrier_init();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_vt);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Number of key tiles item `it` visits (causal items stop at the diagonal).
  auto item_nkv = [&](int item) -> int {
    if (!args.causal) return NKV_ALL;
    const int qt = item % QT;
    const int qend = min(S, qt * 128 + 128);
    return (qend + BN - 1) / BN;
  };

  if (warp == 0) {
    if (lane == 0) {  // ================= TMA producer
      int g = 0, it = 0;
      int lastq[2] = {-1, -1}, lastkv[2] = {-1, -1};
      for (int item = blockIdx.x; item < args.num_items; item += gridDim.x, ++it) {
        const int bh = item / QT, qt = item % QT;
        const int qb = it % C::QST;
        if (!mbar_wait(&q_empty[qb], ((it / C::QST) & 1) ^ 1, wc)) break;
        mbar_arrive_expect_tx(&q_full[qb], C::Q_BYTES);
        for (int kc = 0; kc < C::QKC; ++kc)
          tma_load_3d(sQ + qb * C::Q_BYTES + kc * 128 * C::QKROW, &map_q, &q_full[qb], kc * 64, qt * 128, bh);
        lastq[qb] = it;
        const int nkv = item_nkv(item);
        bool ok = true;
        for (int j = 0; j < nkv; ++j, ++g) {
          const int st = g % C::KVST;
          if (!mbar_wait(&kv_empty[st], ((g / C::KVST) & 1) ^ 1, wc)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[st], C::K_BYTES + C::V_BYTES);
          uint8_t* k_dst = sK + st * C::K_BYTES;
          uint8_t* v_dst = sV + st * C::V_BYTES;
          for (int kc = 0; kc < C::QKC; ++kc)
            tma_load_3d(k_dst + kc * BN * C::QKROW, &map_k, &kv_full[st], kc * 64, j * BN, bh);
          for (int kc = 0; kc < BN / 64; ++kc)
            tma_load_3d(v_dst + kc * DHP * 128, &map_vt, &kv_full[st], j * BN + kc * 64, 0, bh);
          lastkv[st] = g;
        }
        if (!ok) break;
      }
      for (int i = 0; i < 2; ++i) {
        if (lastq[i] >= 0) mbar_drain(&q_full[i], (lastq[i] / C::QST) & 1);
        if (lastkv[i] >= 0) mbar_drain(&kv_full[i], (lastkv[i] / C::KVST) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ================= MMA issuer
      const uint32_t idesc_s = idesc_f16_f32(128, BN);
      const uint32_t idesc_o = idesc_f16_f32(128, DHP);
      const uint32_t t_s = tmem_base + C::S_COL;
      const uint32_t t_o = tmem_base + C::O_COL;
      int g = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x, ++it) {
        const int qb = it % C::QST;
        if (!mbar_wait(&q_full[qb], (it / C::QST) & 1, wc)) break;
        const uint32_t q_base = smem_u32(sQ + qb * C::Q_BYTES);
        const int nkv = item_nkv(item);
        for (int j = 0; j <= nkv; ++j) {
          if (j < nkv) {  // S_j = Q K_j^T
            const int st = (g + j) % C::KVST;
            if (!mbar_wait(&kv_full[st], ((g + j) / C::KVST) & 1, wc)) { ok = false; break; }
            if (g + j > 0 && !mbar_wait(s_free, (g + j - 1) & 1, wc)) { ok = false; break; }
            tc_fence_after();
            const uint32_t k_base = smem_u32(sK + st * C::K_BYTES);
#pragma unroll
            for (int k = 0; k < DHP / 16; ++k) {
              const uint32_t off_q = (uint32_t)((k * 32) / C::QKROW) * (128 * C::QKROW) + (k * 32) % C::QKROW;
              const uint32_t off_k = (uint32_t)((k * 32) / C::QKROW) * (BN * C::QKROW) + (k * 32) % C::QKROW;
              umma_f16_ss(t_s, sdesc_kmajor(q_base + off_q, C::QKROW), sdesc_kmajor(k_base + off_k, C::QKROW),
                          idesc_s, k > 0 ? 1u : 0u);
            }
            umma_commit(s_full);
            if (j == nkv - 1) umma_commit(&q_empty[qb]);
          }
          if (j > 0) {  // O += P_{j-1} V_{j-1}
            const int gp = g + j - 1;
            const int st = gp % C::KVST;
            if (!mbar_wait(p_full, gp & 1, wc)) { ok = false; break; }
            tc_fence_after();
            const uint32_t p_base = smem_u32(sP);
            const uint32_t v_base = smem_u32(sV + st * C::V_BYTES);
#pragma unroll
            for (int k = 0; k < BN / 16; ++k) {
              const uint32_t off_p = (uint32_t)(k >> 2) * 16384 + (k & 3) * 32;
              const uint32_t off_v = (uint32_t)(k >> 2) * (DHP * 128) + (k & 3) * 32;
              umma_f16_ss(t_o, sdesc_kmajor(p_base + off_p, 128), sdesc_kmajor(v_base + off_v, 128), idesc_o,
                          (j > 1 || k > 0) ? 1u : 0u);
            }
            umma_commit(pv_done);
            umma_commit(&kv_empty[st]);
          }
        }
        g += nkv;
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else {  // ================= softmax warps 2..5: one query row per thread
    const int qd = warp & 3;
    const int row = qd * 32 + lane;
    const uint32_t lane_off = (uint32_t)(qd * 32) << 16;
    const uint32_t t_s = tmem_base + lane_off + C::S_COL;
    const uint32_t t_o = tmem_base + lane_off + C::O_COL;
    const uint32_t p_base = smem_u32(sP);
    const float sl2 = args.scale_log2;
    int g = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x) {
      const int bh = item / QT, qt = item % QT;
      const int q0 = qt * 128;
      const int qpos = q0 + row;
      const int nkv = item_nkv(item);
      float m_use = 0.f, l = 0.f;
      const uint8_t* mrow = (KMASK && args.kmask) ? args.kmask + (long long)(bh / args.H) * S : nullptr;
      for (int j = 0; j < nkv; ++j, ++g) {
        uint32_t kb[BN / 32];
        if (KMASK && mrow) key_mask_load<BN / 32>(mrow, j * BN, S, lane, kb);
        if (!mbar_wait(s_full, g & 1, wc)) { ok = false; break; }
        tc_fence_after();
        float s[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(t_s + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free);

        const int kv0 = j * BN;
        const bool need_mask = (kv0 + BN > S) || (args.causal && kv0 + BN - 1 > q0);
        if (need_mask) {
          const int lim = args.causal ? min(S, qpos + 1) : S;  // keys [0, lim) are visible
#pragma unroll
          for (int c = 0; c < BN; ++c)
            if (kv0 + c >= lim) s[c] = -INFINITY;
        }
        if (KMASK && mrow) {   // key padding: invalid keys get probability 0 (-inf score)
          key_mask_ballot<BN / 32>(kb);
          uint32_t all = kb[0];
#pragma unroll
          for (int w = 1; w < BN / 32; ++w) all &= kb[w];
          if (all != 0xffffffffu) {
#pragma unroll
            for (int c = 0; c < BN; ++c)
              if (!((kb[c >> 5] >> (c & 31)) & 1u)) s[c] = -INFINITY;
          }
        }
        float mx = s[0];
#pragma unroll
        for (int c = 1; c < BN; ++c) mx = fmaxf(mx, s[c]);
        const float m_cand = mx * sl2;
        float alpha = 1.f;
        bool rescale = false;
        if (j == 0) {
          m_use = (m_cand == -INFINITY) ? 0.f : m_cand;
        } else if (m_cand > m_use + 8.f) {
          alpha = ex2_approx(m_use - m_cand);
          m_use = m_cand;
          rescale = true;
        }
        float rs = 0.f;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          s[c] = ex2_approx(fmaf(s[c], sl2, -m_use));
          rs += s[c];
        }
        if (j > 0) {
          // P buffer and O are owned by the previous PV MMA until it completes.
          if (!mbar_wait(pv_done, (g - 1) & 1, wc)) { ok = false; break; }
          tc_fence_after();
          if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
            for (int c = 0; c < DHP / 32; ++c) {
              uint32_t r[32];
              tmem_ld32(t_o + c * 32, r);
#pragma unroll
              for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
              tmem_st32(t_o + c * 32, r);
            }
          }
        }
        l = l * alpha + rs;
        // P row -> swizzled fp16 operand tile (atom columns of 64 keys).
#pragma unroll
        for (int c8 = 0; c8 < BN / 8; ++c8) {
          const uint32_t addr = p_base + (uint32_t)(c8 >> 3) * 16384 + swz_offset(row, c8 & 7, 128);
          st_shared_v4(addr, pack_half2(s[8 * c8 + 0], s[8 * c8 + 1]), pack_half2(s[8 * c8 + 2], s[8 * c8 + 3]),
                       pack_half2(s[8 * c8 + 4], s[8 * c8 + 5]), pack_half2(s[8 * c8 + 6], s[8 * c8 + 7]));
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      // ---- epilogue: ctx row = O / l (fp16), rows beyond S are not stored.
      if (!mbar_wait(pv_done, (g - 1) & 1, wc)) { ok = false; break; }
      tc_fence_after();
      const float inv_l = l > 0.f ? 1.0f / l : 0.f;   // a row with every key masked -> 0
      const int b = bh / args.H, h = bh % args.H;
      __half* dst = args.ctx + ((long long)b * S + qpos) * args.d + (long long)h * args.dh;
#pragma unroll 1
      for (int c = 0; c < DHP / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_o + c * 32, r);
        if (qpos < S && c * 32 < args.dh) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            d4[v] = make_uint4(pack_half2(__uint_as_float(r[8 * v + 0]) * inv_l, __uint_as_float(r[8 * v + 1]) * inv_l),
                               pack_half2(__uint_as_float(r[8 * v + 2]) * inv_l, __uint_as_float(r[8 * v + 3]) * inv_l),
                               pack_half2(__uint_as_float(r[8 * v + 4]) * inv_l, __uint_as_float(r[8 * v + 5]) * inv_l),
                               pack_half2(__uint_as_float(r[8 * v + 6]) * inv_l, __uint_as_float(r[8 * v + 7]) * inv_l));
          }
        }
      }
      tc_fence_before();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && waitctl_aborted(wc)) record_error(status, kErrTimeout, kAttn, 0);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

}  // namespace b200l
