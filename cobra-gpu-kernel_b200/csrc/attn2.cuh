// attn2.cuh -- K2 for head_dim <= 64: flash attention with two query tiles
// per CTA, three MMA-issuing warps, sixteen softmax warps, and S, P and O in
// tensor memory.
//
// Same arithmetic as attn.cuh (BaselineSelfAttention.forward,
// torch_transformer_benchmark.py:98-113, without materialising the scores);
// the schedule is built for the long-sequence configs (S up to 100000,
// head_dim 32 / 64). Measured on B200 (one SM, clock64):
//   * one thread issues one M=128 tcgen05.mma per 77-100 cycles whatever N
//     (<= 128), while the tensor core finishes N=128 in ~64 cycles; two
//     threads issuing into different accumulators reach the tensor core's
//     own rate -- so the MMAs are spread over three issuing threads;
//   * the exponentials (FFMA2 -> 2x MUFU ex2 -> FADD2 + fp16 pack per pair of
//     scores) reach 74 % of MUFU throughput with one warp per scheduler, 90 %
//     with two and 96 % with three or four -- so sixteen softmax warps, four
//     per scheduler, each handling 16 rows with two threads per row;
//   * under MUFU load every shared-memory / barrier / TMEM round trip of a
//     warp costs 150-250 cycles, so each warp's step is a short fixed chain
//     of them around its exponentials, and the two halves of a row live in
//     one warp (16x32bx2 TMEM loads / stores: threads 0-15 take keys [0, 64),
//     threads 16-31 keys [64, 128) of the same 16 rows) so that they agree on
//     the row maximum with one shuffle instead of a shared-memory exchange.
// Structure:
//   * a work item is (b, h, 256 queries) = two 128-row query tiles that share
//     every K / v^T tile (one TMA load feeds both tiles' MMAs);
//   * warp 1 issues S = Q K^T for both tiles, warps 2 and 3 issue P v for
//     tile 0 and 1;
//   * warps 4-19 are the softmax: warp 4 + 8t + 4hh + q handles rows
//     32q + 16hh .. 32q + 16hh + 15 of tile t, thread l and l + 16 the two key
//     halves of one row;
//   * per tile, TMEM holds S (fp32, 128 columns), P (fp16 pairs, 64 columns)
//     and O (fp32, dhp columns): the softmax releases S as soon as its rows
//     are in registers, so the next S = Q K^T is computed while the
//     exponentials run; P waits in registers until the previous P v has read
//     the P buffer, and tcgen05.mma reads P from TMEM as its A operand (P
//     never touches shared memory);
//   * K / v^T stream through a 3-stage TMA ring; lazy rescaling of O (only when
//     a row max grows by more than 2^8; each thread rescales its half of O).
// TMEM (512 columns): S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384)
// O0 [384, 384+dhp) O1 [448, 448+dhp).
// S issuer, per key tile j and tile t: S_t(j) once the eight softmax warps of
// tile t have read S_t(j-1) (and K tile j has landed). P v issuer t: P_t(j)
// v_j once they have written P_t(j).
#pragma once

#include "attn.cuh"
#include "common.cuh"

namespace b200l {

template <int DHP>
struct Attn2Cfg {
  static constexpr int BN = 128;
  static constexpr int QKROW = DHP >= 64 ? 128 : 64;   // bytes per swizzled Q/K row
  static constexpr int QKC = DHP * 2 / QKROW;          // atom columns along dh
  static constexpr int Q_BYTES = 128 * DHP * 2;        // one query tile
  static constexpr int K_BYTES = BN * DHP * 2;
  static constexpr int V_BYTES = DHP * BN * 2;         // v^T tile: DHP rows x 128 keys
  static constexpr int KVST = 3;
  static constexpr int SMEM = 2 * Q_BYTES + KVST * (K_BYTES + V_BYTES) + 256 + 1024;
  static constexpr int THREADS = 640;
  static constexpr int S_COL = 0;      // + 128 * t
  static constexpr int P_COL = 256;    // + 64 * t
  static constexpr int O_COL = 384;    // + 64 * t
};

template <int DHP, bool KMASK>   // KMASK: a key-padding mask may be given
__global__ void __launch_bounds__(640, 1)
    attn2_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                 const __grid_constant__ CUtensorMap map_vt, AttnArgs args, DevStatus* status) {
  pdl_wait_then_release();
  using C = Attn2Cfg<DHP>;
  constexpr int BN = C::BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // Q0 | Q1
  uint8_t* sK = sQ + 2 * C::Q_BYTES;
  uint8_t* sV = sK + C::KVST * C::K_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + C::KVST * C::V_BYTES);
  uint64_t* q_full = bars;
  uint64_t* q_empty = bars + 1;    // the S issuer releases Q after the item's last S
  uint64_t* kv_full = bars + 2;    // [3]
  uint64_t* kv_empty = bars + 5;   // [3] both P v issuers release a stage after their P v of it
  uint64_t* s_full = bars + 8;     // [2] per tile: S_t in TMEM
  uint64_t* s_free = bars + 10;    // [2] per tile: the softmax warps have read S_t
  uint64_t* p_full = bars + 12;    // [2] per tile: P_t written to TMEM
  uint64_t* pv_done = bars + 14;   // [2] per tile: P_t v complete (P_t and O_t free)
  uint64_t* mma_done = bars + 16;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 17);
  WaitCtl* wc = reinterpret_cast<WaitCtl*>(bars + 18);   // bars 18-19

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = args.S;
  const int QP = (S + 255) / 256;                       // query pairs per (b, h)
  const int num_items = args.B * args.H * QP;
  const int NKV_ALL = (S + BN - 1) / BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_free[t], 8);
      mbar_init(&p_full[t], 8);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(mma_done, 3);
    waitctl_init(wc, status);
    fence_barrier_init();
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_vt);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  // Query tiles an item has (the second one may lie entirely past S) and the
  // key tiles it visits (causal items stop after their last query).
  auto item_nqt = [&](int item) -> int { return (S - (item % QP) * 256) > 128 ? 2 : 1; };
  auto item_nkv = [&](int item) -> int {
    if (!args.causal) return NKV_ALL;
    const int qend = min(S, (item % QP) * 256 + 256);
    return (qend + BN - 1) / BN;
  };

  if (warp == 0) {
    if (lane == 0) {  // ================= TMA producer
      int g = 0, it = 0, lastkv[3] = {-1, -1, -1}, lastq = -1;
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x, ++it) {
        const int bh = item / QP, q0 = (item % QP) * 256;
        const int nqt = item_nqt(item);
        if (!mbar_wait(q_empty, (it & 1) ^ 1, wc)) break;
        mbar_arrive_expect_tx(q_full, nqt * C::Q_BYTES);
        for (int t = 0; t < nqt; ++t)
          for (int kc = 0; kc < C::QKC; ++kc)
            tma_load_3d(sQ + t * C::Q_BYTES + kc * 128 * C::QKROW, &map_q, q_full, kc * 64, q0 + t * 128, bh);
        lastq = it;
        const int nkv = item_nkv(item);
        for (int j = 0; j < nkv; ++j, ++g) {
          const int st = g % C::KVST;
          if (!mbar_wait(&kv_empty[st], ((g / C::KVST) & 1) ^ 1, wc)) { ok = false; break; }
          // Test hook: CTA 0 leaves out its first K / v^T load (nothing issued,
          // so nothing to drain); the MMA issuers' bounded waits run out.
          if (g == 0 && blockIdx.x == 0 && wc->site == kSiteAttnKv) continue;
          mbar_arrive_expect_tx(&kv_full[st], C::K_BYTES + C::V_BYTES);
          for (int kc = 0; kc < C::QKC; ++kc)
            tma_load_3d(sK + st * C::K_BYTES + kc * BN * C::QKROW, &map_k, &kv_full[st], kc * 64, j * BN, bh);
          for (int kc = 0; kc < BN / 64; ++kc)
            tma_load_3d(sV + st * C::V_BYTES + kc * DHP * 128, &map_vt, &kv_full[st], j * BN + kc * 64, 0, bh);
          lastkv[st] = g;
        }
      }
      if (lastq >= 0) mbar_drain(q_full, lastq & 1);
      for (int i = 0; i < 3; ++i)
        if (lastkv[i] >= 0) mbar_drain(&kv_full[i], (lastkv[i] / C::KVST) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ================= S issuer: S_t(j) = Q_t K_j^T for both tiles
      const uint32_t idesc_s = idesc_f16_f32(128, BN);
      // Shared-memory descriptors of Q0 and of the first K stage; every other
      // operand is a fixed byte offset away, added to the start-address field
      // (addresses stay below 256 KB, so it never carries).
      const uint64_t dq0 = sdesc_kmajor(smem_u32(sQ), C::QKROW);
      const uint64_t dk0 = sdesc_kmajor(smem_u32(sK), C::QKROW);
      // g: key tiles so far (ring stage); ns[t]: S steps of tile t so far.
      int g = 0, it = 0, ns[2] = {0, 0};
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x, ++it) {
        const int nqt = item_nqt(item);
        const int nkv = item_nkv(item);
        if (!mbar_wait(q_full, it & 1, wc)) break;
        for (int j = 0; j < nkv && ok; ++j) {
          const int st = (g + j) % C::KVST;
          if (!mbar_wait(&kv_full[st], ((g + j) / C::KVST) & 1, wc)) { ok = false; break; }
          const uint64_t dk = dk0 + (uint64_t)((st * C::K_BYTES) >> 4);
          for (int t = 0; t < nqt; ++t) {
            // S_t is free once softmax t has read the previous S_t.
            if (ns[t] > 0 && !mbar_wait(&s_free[t], (ns[t] - 1) & 1, wc)) { ok = false; break; }
            const uint64_t dq = dq0 + (uint64_t)((t * C::Q_BYTES) >> 4);
            const uint32_t d_s = tmem_base + C::S_COL + t * 128;
            tc_fence_after();
#pragma unroll
            for (int k = 0; k < DHP / 16; ++k) {
              constexpr int R = C::QKROW;
              const uint32_t off_q = (uint32_t)((k * 32) / R) * (128 * R) + (k * 32) % R;
              const uint32_t off_k = (uint32_t)((k * 32) / R) * (BN * R) + (k * 32) % R;
              umma_f16_ss(d_s, dq + (off_q >> 4), dk + (off_k >> 4), idesc_s, k > 0 ? 1u : 0u);
            }
            umma_commit(&s_full[t]);
            ++ns[t];
          }
        }
        if (ok) umma_commit(q_empty);   // after the item's last S: Q may be reloaded
        g += nkv;
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else if (warp == 2 || warp == 3) {
    if (lane == 0) {  // ================= P v issuer of query tile t: O_t += P_t(j) v_j
      const int t = warp - 2;
      const uint32_t idesc_o = idesc_f16_f32(128, DHP);
      const uint64_t dv0 = sdesc_kmajor(smem_u32(sV), 128);
      const uint32_t a_p = tmem_base + C::P_COL + t * 64;
      const uint32_t d_o = tmem_base + C::O_COL + t * 64;
      // g: key tiles so far (ring stage); np: P v steps of this tile so far.
      int g = 0, np = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
        const int nqt = item_nqt(item);
        const int nkv = item_nkv(item);
        for (int j = 0; j < nkv && ok; ++j) {
          const int st = (g + j) % C::KVST;
          if (t >= nqt) {
            // No second query tile in this item: release each K / v^T stage
            // once it has landed (so this issuer never arrives on a stage
            // ahead of the other one).
            if (!mbar_wait(&kv_full[st], ((g + j) / C::KVST) & 1, wc)) { ok = false; break; }
            umma_commit(&kv_empty[st]);
            continue;
          }
          // P_t(j) in TMEM (softmax t read S_t(j), so K / v^T tile j has landed).
          if (!mbar_wait(&p_full[t], np & 1, wc)) { ok = false; break; }
          const uint64_t dv = dv0 + (uint64_t)((st * C::V_BYTES) >> 4);
          const uint32_t acc0 = j > 0 ? 1u : 0u;
          tc_fence_after();
#pragma unroll
          for (int k = 0; k < BN / 16; ++k)
            umma_f16_ts(d_o, a_p + k * 8, dv + ((uint32_t)((k >> 2) * (DHP * 128) + (k & 3) * 32) >> 4), idesc_o,
                        k > 0 ? 1u : acc0);
          umma_commit(&pv_done[t]);
          umma_commit(&kv_empty[st]);
          ++np;
        }
        g += nkv;
      }
      umma_commit(mma_done);
      mbar_drain(mma_done, 0);
    }
  } else {  // ================= softmax: tile t, 16 query rows per warp, two threads per row
    // Warp 4 + 8t + 4hh + qd handles rows 32qd + 16hh .. + 15 of tile t: the
    // 16x32bx2 TMEM forms give threads 0-15 keys [0, 64) and threads 16-31
    // keys [64, 128) of the same 16 rows, so the two halves of a row are
    // lanes l and l + 16 of one warp and agree on the row maximum (and, at
    // the end, the row sum) with one shuffle.
    const int sw = warp - 4;
    const int t = sw >> 3;
    const int hh = (sw >> 2) & 1;
    const int qd = warp & 3;
    const int c = lane >> 4;                       // key half of this thread
    const int row = qd * 32 + hh * 16 + (lane & 15);
    const uint32_t lane_off = (uint32_t)(qd * 32 + hh * 16) << 16;
    const uint32_t t_s = tmem_base + lane_off + C::S_COL + t * 128;
    const uint32_t t_p = tmem_base + lane_off + C::P_COL + t * 64;
    constexpr int OH = DHP / 2;                    // O columns of this thread: [OH c, OH c + OH)
    const uint32_t t_o = tmem_base + lane_off + C::O_COL + t * 64;
    const int ocol0 = OH * c;
    const float sl2 = args.scale_log2;
    int ns = 0, np = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < num_items && ok; item += gridDim.x) {
      const int nqt = item_nqt(item);
      const int nkv = item_nkv(item);
      if (t >= nqt) continue;
      const int bh = item / QP;
      const int q0 = (item % QP) * 256 + t * 128;
      const int qpos = q0 + row;
      const int lim = args.causal ? min(S, qpos + 1) : S;   // keys [0, lim) are visible
      float m_use = 0.f, l = 0.f;
      const uint8_t* mrow = (KMASK && args.kmask) ? args.kmask + (long long)(bh / args.H) * S : nullptr;
      for (int j = 0; j < nkv; ++j) {
        const int kv0 = j * BN + 64 * c;   // first key of this thread's half
        uint32_t kb[4];
        if (KMASK && mrow) key_mask_load<4>(mrow, j * BN, S, lane, kb);
        if (!mbar_wait_warp(&s_full[t], ns & 1, wc)) { ok = false; break; }
        tc_fence_after();
        float s[64];
        {
          uint32_t r[64];
          tmem_ld_pair64<64>(t_s, r);
#pragma unroll
          for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(r[i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[t]);
        ++ns;
        if (__any_sync(0xffffffffu, (kv0 + 64 > S) || (args.causal && kv0 + 63 > q0))) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (kv0 + i >= lim) s[i] = -INFINITY;
        }
        if (KMASK && mrow) {
          key_mask_ballot<4>(kb);
          if ((kb[0] & kb[1] & kb[2] & kb[3]) != 0xffffffffu) {
            const uint32_t k0 = c ? kb[2] : kb[0], k1 = c ? kb[3] : kb[1];
#pragma unroll
            for (int i = 0; i < 64; ++i)
              if (!(((i < 32 ? k0 : k1) >> (i & 31)) & 1u)) s[i] = -INFINITY;
          }
        }
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = fmaxf(s[2 * k], s[2 * k + 1]);
#pragma unroll
        for (int i = 8; i < 32; ++i) m8[i & 7] = fmax3f(m8[i & 7], s[2 * i], s[2 * i + 1]);
        const float hm = fmax3f(fmax3f(m8[0], m8[1], m8[2]), fmax3f(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        const float mx = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, 16));
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
        const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-m_use, -m_use);
        // head_dim 32: the previous P v (P buffer, and O for a rescale) has
        // usually completed by now, so its phase is tested before the
        // exponentials (the test's latency hides under them) and waited for
        // below only if it had not (cfg4 attention 0.107 -> 0.101 ms). At
        // head_dim 64 P v takes twice as long and the early test measured
        // 1.5 % slower, so there the wait stays where P is stored.
        constexpr bool kEarlyPvTest = DHP <= 32;
        const bool pv_seen = (np == 0) || (kEarlyPvTest && mbar_test_wait(&pv_done[t], (np - 1) & 1));
        float2 acc[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                         make_float2(0.f, 0.f)};
        uint32_t pk[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float2 xx = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), sc2, nm2);
          const float2 pp = make_float2(ex2_approx(xx.x), ex2_approx(xx.y));
          acc[i & 3] = __fadd2_rn(acc[i & 3], pp);
          pk[i] = pack_half2(pp.x, pp.y);
        }
        const float2 a01 = __fadd2_rn(acc[0], acc[1]), a23 = __fadd2_rn(acc[2], acc[3]);
        l = l * alpha + ((a01.x + a01.y) + (a23.x + a23.y));
        if (np > 0) {
          if (!__all_sync(0xffffffffu, pv_seen) && !mbar_wait_warp(&pv_done[t], (np - 1) & 1, wc)) {
            ok = false;
            break;
          }
          tc_fence_after();
        }
        if (j > 0 && __any_sync(0xffffffffu, rescale)) {
          uint32_t r[OH];
          if constexpr (OH == 16) tmem_ld_pair16<16>(t_o, *reinterpret_cast<uint32_t(*)[16]>(r));
          else tmem_ld_pair32<32>(t_o, *reinterpret_cast<uint32_t(*)[32]>(r));
#pragma unroll
          for (int i = 0; i < OH; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * alpha);
          if constexpr (OH == 16) tmem_st_pair16<16>(t_o, *reinterpret_cast<uint32_t(*)[16]>(r));
          else tmem_st_pair32<32>(t_o, *reinterpret_cast<uint32_t(*)[32]>(r));
        }
        tmem_st_pair32<32>(t_p, pk);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
        ++np;
      }
      if (!ok) break;
      // ---- epilogue: the two halves' row sums, then ctx = O / l (fp16).
      if (!mbar_wait_warp(&pv_done[t], (np - 1) & 1, wc)) { ok = false; break; }
      const float lt = l + __shfl_xor_sync(0xffffffffu, l, 16);
      tc_fence_after();
      const float inv_l = lt > 0.f ? 1.0f / lt : 0.f;
      const int b = bh / args.H, h = bh % args.H;
      uint32_t r[OH];
      if constexpr (OH == 16) tmem_ld_pair16<16>(t_o, *reinterpret_cast<uint32_t(*)[16]>(r));
      else tmem_ld_pair32<32>(t_o, *reinterpret_cast<uint32_t(*)[32]>(r));
      if (qpos < S && ocol0 < args.dh) {
        __half* dst = args.ctx + ((long long)b * S + qpos) * args.d + (long long)h * args.dh + ocol0;
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int v = 0; v < OH / 8; ++v) {
          d4[v] = make_uint4(pack_half2(__uint_as_float(r[8 * v + 0]) * inv_l, __uint_as_float(r[8 * v + 1]) * inv_l),
                             pack_half2(__uint_as_float(r[8 * v + 2]) * inv_l, __uint_as_float(r[8 * v + 3]) * inv_l),
                             pack_half2(__uint_as_float(r[8 * v + 4]) * inv_l, __uint_as_float(r[8 * v + 5]) * inv_l),
                             pack_half2(__uint_as_float(r[8 * v + 6]) * inv_l, __uint_as_float(r[8 * v + 7]) * inv_l));
        }
      }
      tc_fence_before();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && waitctl_aborted(wc)) record_error(status, kErrTimeout, kAttn, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace b200l
