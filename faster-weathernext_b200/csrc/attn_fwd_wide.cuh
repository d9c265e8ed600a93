// Forward kernel for dense neighbourhoods (bf16, 128-row tile lists): 128-key chunks.
//
// Same math as attn_fwd.cuh (the Pallas-Triton `_kernel`, src/faster_weathernext/pallas_attn.py:112-141):
// per query row an online softmax over the allowed keys of its block's active 32-key tiles, masked logits
// contributing exactly 0, O = acc / l, LSE = m + log(l).
//
// Why a second kernel: a tcgen05.mma instruction (M = 128, K = 16) takes about as long for N = 32 as for
// N = 128, so S = Q K^T over 32- or 64-key chunks leaves most of the tensor core idle once the mask is
// dense (the WeatherNext 2 32-hop mask: 3,101 keys per query, ~190 tiles per 128-row block). Here a chunk
// is four consecutive tiles of the list (up to 128 keys): S MMAs have N = 128 and P V has K = 128.
//
// Work item = (batch, head, 128-query block); persistent CTAs, one per SM. TMEM (512 columns): S[2]
// (128 each), O (D), P[2] (64 each: 128 bf16 keys). Shared memory: Q, a ring of K tiles (released when
// S is done), a ring of V tiles (released when P V is done), a ring of mask words. Roles (320 threads):
//   warp 0      TMA producer: Q once per item; per chunk K, the mask words, then V of the previous chunk.
//               Four tiles with consecutive key blocks are one 128-row box per column block, otherwise
//               one 32-row box per tile; copies are issued from several lanes at once.
//   warp 1      TMEM allocation; the warp runs the MMA loop (descriptors warp-uniform) and one elected lane
//               issues S = Q K^T (A, B from shared memory) into S[c & 1] and O += P V (A = P from TMEM,
//               B = V MN-major); S of chunk c+1 goes ahead of P V of chunk c.
//   warps 2-9   softmax. Warps w and w+4 share TMEM lane quadrant w % 4 (thread = query row) and take
//               columns 0-63 and 64-127 of each chunk. One pass against the row's reference max (the exact
//               masked max of the first chunk with an allowed key); if a half-row's sum exceeds 2^8 the
//               pair redoes the chunk with the exact two-pass update (and rescales O in TMEM). The two
//               warps of a pair exchange maxima, flags and sums through shared memory and an mbarrier.
//               P (bf16) goes to TMEM. Epilogue: O / l (each warp its half of the columns) and LSE.
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA drains and returns with the device
// error word set.
#pragma once

#include <cuda.h>

#include "attn_fwd.cuh"
#include "common.cuh"

namespace fwn {

template <int D>
struct WideCfg {
  static constexpr int ES = 2;
  static constexpr int EPB = 64;              // bf16 elements per 128-byte column block
  static constexpr int CB = D / EPB;
  static constexpr int ROWS = 128;
  static constexpr int SUB = 32;
  static constexpr int CH = 4;                // tiles per chunk
  static constexpr int KEYS = SUB * CH;
  static constexpr int Q_BYTES = CB * ROWS * 128;
  static constexpr int KV_BYTES = CB * KEYS * 128;  // one K or V chunk
  static constexpr int NK = D == 128 ? 3 : 4;       // K ring
  static constexpr int NV = D == 128 ? 2 : 3;       // V ring
  static constexpr int NBB = 4;                     // mask-word ring (CH * 512 bytes per chunk)
  static constexpr int OFF_K = Q_BYTES;
  static constexpr int OFF_V = OFF_K + NK * KV_BYTES;
  static constexpr int OFF_BITS = OFF_V + NV * KV_BYTES;
  static constexpr int OFF_X = OFF_BITS + NBB * CH * 512;
  // Pair exchange: 2 slots x {fresh max, two-pass max, sum} x 2 halves x 128 rows floats, + flags.
  static constexpr int X_BYTES = 2 * 3 * 2 * 128 * 4 + 2 * 2 * 4 * 4;
  static constexpr int OFF_BAR = OFF_X + X_BYTES;
  static constexpr int N_BAR = 2 + 2 * NK + 2 * NV + 2 * NBB + 4 + 4 + 3 + 4;
  static constexpr int SMEM_BYTES = OFF_BAR + N_BAR * 8 + 16 + 1024;
  static constexpr int O_COL = 2 * KEYS;
  static constexpr int P_COL = O_COL + D;           // P[b] at P_COL + 64 b
  static constexpr int TMEM_COLS = 512;
  static constexpr int THREADS = 320;
  static constexpr int POLY_PAIRS = 1;              // of the 4 column pairs of a group of 8: polynomial 2^x
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(P_COL + 128 <= TMEM_COLS, "TMEM budget");
  static_assert(D % EPB == 0, "head_dim must fill whole 128-byte column blocks");
};

template <int D>
// Registers: each of an SM's four sub-partitions holds 16,384; ten warps put three on two of them, so at most
// 168 per thread (the runtime refuses the launch above that).
__global__ void __maxnreg__(168)
    attn_fwd_wide_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_k4,
                         const __grid_constant__ CUtensorMap tm_v4, const FwdParams p) {
  using C = WideCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_smem = sbase;
  auto k_slot = [&](int s) { return sbase + C::OFF_K + s * C::KV_BYTES; };
  auto v_slot = [&](int s) { return sbase + C::OFF_V + s * C::KV_BYTES; };
  auto bits_slot = [&](int s) { return sbase + C::OFF_BITS + s * C::CH * 512; };
  float* xch = reinterpret_cast<float*>(smem + C::OFF_X);  // [slot 2][kind 3][half 2][row 128]
  int* xflag = reinterpret_cast<int*>(smem + C::OFF_X + 2 * 3 * 2 * 128 * 4);  // [slot 2][half 2][quadrant 4]
  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t q_full = bar0, q_empty = bar0 + 8;
  auto k_full = [&](int s) { return bar0 + 16 + 8 * s; };
  auto k_empty = [&](int s) { return bar0 + 16 + 8 * (C::NK + s); };
  const uint32_t bar1 = bar0 + 16 + 16 * C::NK;
  auto v_full = [&](int s) { return bar1 + 8 * s; };
  auto v_empty = [&](int s) { return bar1 + 8 * (C::NV + s); };
  const uint32_t bar2 = bar1 + 16 * C::NV;
  auto b_full = [&](int s) { return bar2 + 8 * s; };
  auto b_empty = [&](int s) { return bar2 + 8 * (C::NBB + s); };
  const uint32_t bar3 = bar2 + 16 * C::NBB;
  auto s_full = [&](int b) { return bar3 + 8 * b; };
  auto s_empty = [&](int b) { return bar3 + 16 + 8 * b; };
  auto p_full = [&](int b) { return bar3 + 32 + 8 * b; };
  auto p_empty = [&](int b) { return bar3 + 48 + 8 * b; };
  const uint32_t o_full = bar3 + 64, o_empty = bar3 + 72, drain = bar3 + 80;
  auto pair_bar = [&](int quadrant) { return bar3 + 88 + 8 * quadrant; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + C::N_BAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + C::N_BAR * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int trace_count = 0;  // FWN_TRACE builds: this lane's event count
#define FWN_TR(code, arg) trace_event(p.trace, trace_count, (code), (arg))
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::NK; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < C::NV; ++s) {
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int s = 0; s < C::NBB; ++s) {
      mbar_init(b_full(s), 1);
      mbar_init(b_empty(s), 8);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(s_empty(b), 8);
      mbar_init(p_full(b), 8);
      mbar_init(p_empty(b), 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, 8);
    mbar_init(drain, 1);
    for (int q = 0; q < 4; ++q) mbar_init(pair_bar(q), 2);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_k4);
    tma_prefetch_desc(&tm_v4);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  const int per_bh = p.np;
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    // nk / nv: K / V chunk copies issued so far (the mask words travel with K): copy i uses slot i % N.
    uint32_t nk = 0, nv = 0, qc = 0;
    bool ok = true;
    int pending_q = 0;
    int it = blockIdx.x;
    int nt0 = 0, nt1 = 0;
    if (it < p.n_items) {
      nt0 = __ldg(p.ptr2 + it % per_bh);
      nt1 = __ldg(p.ptr2 + it % per_bh + 1);
    }
    for (; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh, bh = it / per_bh, h = bh % p.heads, b = bh / p.heads;
      const int t0 = nt0, n_sub = nt1 - nt0;
      const int it_next = it + gridDim.x;
      if (it_next < p.n_items) {
        nt0 = __ldg(p.ptr2 + it_next % per_bh);
        nt1 = __ldg(p.ptr2 + it_next % per_bh + 1);
      }
      const int nch = (n_sub + C::CH - 1) / C::CH;
      if (nch == 0) continue;
      // Lane s (< 4) holds the key block of tile s of a chunk.
      auto meta = [&](int c) { const int i = C::CH * c + (lane & 3); return i < n_sub ? __ldg(p.kb2 + t0 + i) : 0; };
      if (!(ok = mbar_wait(q_empty, (qc & 1) ^ 1, abort_flag))) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, C::Q_BYTES);
        for (int cb = 0; cb < C::CB; ++cb)
          tma_load_4d(q_smem + cb * C::ROWS * 128, &tm_q, cb * C::EPB, h, pb * C::ROWS, b, q_full);
      }
      pending_q = 1;
      // K or V of one chunk into `dst`: one 128-row box per column block for four consecutive tiles, else
      // one 32-row box per tile and column block, issued by lanes 0 .. n_in * CB - 1.
      auto load_op = [&](uint32_t dst, const CUtensorMap* t32, const CUtensorMap* t128, int kbl, int n_in,
                         uint32_t bar) {
        const int k0 = __shfl_sync(0xffffffffu, kbl, 0), k1 = __shfl_sync(0xffffffffu, kbl, 1);
        const int k2 = __shfl_sync(0xffffffffu, kbl, 2), k3 = __shfl_sync(0xffffffffu, kbl, 3);
        const bool run = n_in == 4 && k1 == k0 + 1 && k2 == k0 + 2 && k3 == k0 + 3;
        if (lane == 0) mbar_arrive_expect_tx(bar, n_in * C::SUB * D * C::ES);
        __syncwarp();
        if (run) {
          if (lane < C::CB) tma_load_4d(dst + lane * C::KEYS * 128, t128, lane * C::EPB, h, k0 * C::SUB, b, bar);
        } else if (lane < n_in * C::CB) {
          const int s = lane / C::CB, cb = lane % C::CB;
          const int kb = s == 0 ? k0 : s == 1 ? k1 : s == 2 ? k2 : k3;
          tma_load_4d(dst + cb * C::KEYS * 128 + s * C::SUB * 128, t32, cb * C::EPB, h, kb * C::SUB, b, bar);
        }
      };
      int kb_cur = meta(0), kb_prev = 0;
      for (int c = 0; c <= nch && ok; ++c) {
        const int kb_next = c + 1 < nch ? meta(c + 1) : 0;
        if (c < nch) {
          // K and mask words of chunk c.
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (!(ok = mbar_wait(k_empty(nk % C::NK), ((nk / C::NK) & 1) ^ 1, abort_flag))) break;
          if (!(ok = mbar_wait(b_empty(nk % C::NBB), ((nk / C::NBB) & 1) ^ 1, abort_flag))) break;
          if (lane == 0) FWN_TR(3, c);
          load_op(k_slot(nk % C::NK), &tm_k, &tm_k4, kb_cur, n_in, k_full(nk % C::NK));
          if (lane == 0) {
            mbar_arrive_expect_tx(b_full(nk % C::NBB), n_in * 512);
            bulk_load(bits_slot(nk % C::NBB), p.bits2 + static_cast<size_t>(t0 + C::CH * c) * 128, n_in * 512,
                      b_full(nk % C::NBB));
          }
          ++nk;
        }
        if (c >= 1) {
          // V of chunk c-1 (needed one chunk later than its K).
          const int n_in = min(C::CH, n_sub - C::CH * (c - 1));
          if (!(ok = mbar_wait(v_empty(nv % C::NV), ((nv / C::NV) & 1) ^ 1, abort_flag))) break;
          load_op(v_slot(nv % C::NV), &tm_v, &tm_v4, kb_prev, n_in, v_full(nv % C::NV));
          ++nv;
        }
        kb_prev = kb_cur;
        kb_cur = kb_next;
      }
      if (!ok) break;
      ++qc;
    }
    if (!ok && lane == 0) {
      // Drain: wait (bounded, ignoring the abort flag) for the copies that may still be in flight.
      volatile int never = 0;
      for (uint32_t k = (nk >= C::NK ? nk - C::NK : 0); k < nk; ++k) mbar_wait(k_full(k % C::NK), (k / C::NK) & 1, &never);
      for (uint32_t k = (nk >= C::NBB ? nk - C::NBB : 0); k < nk; ++k)
        mbar_wait(b_full(k % C::NBB), (k / C::NBB) & 1, &never);
      for (uint32_t k = (nv >= C::NV ? nv - C::NV : 0); k < nv; ++k) mbar_wait(v_full(k % C::NV), (k / C::NV) & 1, &never);
      if (pending_q) mbar_wait(q_full, (qc & 1), &never);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (whole warp, one lane issues)
    constexpr uint32_t kIdescPV = instr_desc(false, 128, D, false, true);
    const uint64_t qdesc = smem_desc(q_smem, 16, 1024);
    uint32_t g = 0, qc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh;
      const int t0 = p.ptr2[pb], n_sub = p.ptr2[pb + 1] - t0;
      const int nch = (n_sub + C::CH - 1) / C::CH;
      if (nch == 0) continue;
      if (!(ok = warp_wait(q_full, qc & 1, abort_flag))) break;
      const uint32_t g0 = g;
      for (int c = 0; c <= nch && ok; ++c) {
        if (c < nch) {
          const uint32_t gg = g0 + c;
          const int sb = gg & 1;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (!(ok = warp_wait(k_full(gg % C::NK), (gg / C::NK) & 1, abort_flag))) break;
          if (!(ok = warp_wait(s_empty(sb), ((gg >> 1) & 1) ^ 1, abort_flag))) break;
          if (lane == 0) FWN_TR(13, c);
          tc_fence_after();
          const uint32_t idesc_s = instr_desc(false, 128, 32 * n_in, false, false);
          const uint64_t kdesc = smem_desc(k_slot(gg % C::NK), 16, 1024);
          if (elect_one_sync()) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t cb = kk / 4, within = (kk % 4) * 32;
              mma_ss<false>(tmem + sb * C::KEYS, qdesc + ((cb * C::ROWS * 128 + within) >> 4),
                            kdesc + ((cb * C::KEYS * 128 + within) >> 4), idesc_s, kk > 0 ? 1u : 0u);
            }
            mma_commit(s_full(sb));
            mma_commit(k_empty(gg % C::NK));
            if (c == nch - 1) mma_commit(q_empty);
          }
          __syncwarp();
          if (lane == 0) FWN_TR(11, c);
        }
        if (c >= 1) {
          const uint32_t gg = g0 + c - 1;
          const int pbuf = gg & 1;
          const int n_in = min(C::CH, n_sub - C::CH * (c - 1));
          if (!(ok = warp_wait(p_full(pbuf), (gg >> 1) & 1, abort_flag))) break;
          if (!(ok = warp_wait(v_full(gg % C::NV), (gg / C::NV) & 1, abort_flag))) break;
          if (c == 1 && !(ok = warp_wait(o_empty, (qc & 1) ^ 1, abort_flag))) break;
          if (lane == 0) FWN_TR(14, c - 1);
          tc_fence_after();
          const uint64_t vdesc = smem_desc(v_slot(gg % C::NV), C::KEYS * 128, 1024);
          const uint32_t pcol = tmem + C::P_COL + 64 * pbuf;
          const int ksteps = 2 * n_in;
          if (elect_one_sync()) {
            for (int kk = 0; kk < ksteps; ++kk)
              mma_ts(tmem + C::O_COL, pcol + 8 * kk, vdesc + ((kk * 16 * 128) >> 4), kIdescPV,
                     (c == 1 && kk == 0) ? 0u : 1u);
            mma_commit(p_empty(pbuf));
            mma_commit(v_empty(gg % C::NV));
            if (c == nch) mma_commit(o_full);
          }
          __syncwarp();
          if (lane == 0) FWN_TR(12, c - 1);
        }
      }
      g = g0 + nch;
      ++qc;
    }
    if (elect_one_sync()) mma_commit(drain);
    __syncwarp();
    volatile int never = 0;
    mbar_wait(drain, 0, &never);
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 2-9)
    const int quarter = warp & 3, half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float c2 = p.scale_log2;
    const uint32_t xbar = pair_bar(quarter);
    uint32_t xk = 0;  // pair exchanges done (phase of xbar)
    // Exchange one float per row with the partner warp: returns the partner's value.
    auto exchange = [&](int kind, float v, float& other) -> bool {
      float* slot = xch + (static_cast<int>(xk & 1) * 3 + kind) * 256;
      slot[half * 128 + row] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      if (!mbar_wait(xbar, xk & 1, abort_flag)) return false;
      other = slot[(1 - half) * 128 + row];
      ++xk;
      return true;
    };
    auto exchange_flag = [&](int v, int& other) -> bool {
      int* slot = xflag + static_cast<int>(xk & 1) * 8;
      if (lane == 0) slot[half * 4 + quarter] = v;
      __syncwarp();
      if (lane == 0) mbar_arrive(xbar);
      if (!mbar_wait(xbar, xk & 1, abort_flag)) return false;
      other = slot[(1 - half) * 4 + quarter];
      ++xk;
      return true;
    };
    uint32_t g = 0, qc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh, bh = it / per_bh, h = bh % p.heads, b = bh / p.heads;
      const int t0 = p.ptr2[pb], n_sub = p.ptr2[pb + 1] - t0;
      const int nch = (n_sub + C::CH - 1) / C::CH;
      const int qrow = pb * C::ROWS + row;
      float m_ref = -INFINITY, l = 0.f;   // m_ref is the same in both halves; l is this half's sum
      const uint32_t g0 = g;
      for (int c = 0; c < nch; ++c) {
        const uint32_t gg = g0 + c;
        const int sb = gg & 1, bs = gg % C::NBB;
        const int n_in = min(C::CH, n_sub - C::CH * c);
        const int j0 = 2 * half;  // this half's first tile of the chunk
        // S columns of this half -> registers; the S buffer is free for the next S MMA right away.
        if (!(ok = mbar_wait(s_full(sb), (gg >> 1) & 1, abort_flag))) break;
        if (lane == 0) FWN_TR(20, c);
        tc_fence_after();
        float s[64];
        if (j0 < n_in) tmem_ld32(trow + sb * C::KEYS + 64 * half, *reinterpret_cast<float(*)[32]>(&s[0]));
        if (j0 + 1 < n_in) tmem_ld32(trow + sb * C::KEYS + 64 * half + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty(sb));
        if (!(ok = mbar_wait(b_full(bs), (gg / C::NBB) & 1, abort_flag))) break;
        const uint32_t w0 = j0 < n_in ? ld_shared_u32(bits_slot(bs) + j0 * 512 + row * 4) : 0u;
        const uint32_t w1 = j0 + 1 < n_in ? ld_shared_u32(bits_slot(bs) + (j0 + 1) * 512 + row * 4) : 0u;
        __syncwarp();
        if (lane == 0) mbar_arrive(b_empty(bs));
        const uint32_t a0 = __reduce_or_sync(0xffffffffu, w0), a1 = __reduce_or_sync(0xffffffffu, w1);
        auto half_max = [&]() -> float {
          float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const uint32_t w = i < 32 ? w0 : w1;
            mx[i & 3] = (w >> (i & 31)) & 1u ? fmaxf(mx[i & 3], s[i]) : mx[i & 3];
          }
          return fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        };
        // p = 2^(s c2 - m) for allowed columns (0 elsewhere), packed bf16 pairs into pk; returns the sum.
        // The first pair of each group of 8 columns goes through the FMA-pipe polynomial, the others
        // through MUFU.EX2.
        uint32_t pk[32];
        auto exps = [&](float m) -> float {
          const float2 cc = make_float2(c2, c2), nm = make_float2(-m, -m);
          float2 acc[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
          for (int gi = 0; gi < 8; ++gi) {
            const uint32_t w = gi < 4 ? w0 : w1;
            const uint32_t a = gi < 4 ? a0 : a1;
            if ((a >> (8 * (gi & 3))) & 0xFFu) {
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const int k = 8 * gi + i;
                const float2 x = ffma2(make_float2(s[k], s[k + 1]), cc, nm);
                float2 e;
                if (i < C::POLY_PAIRS * 2) {
                  e = exp2_poly2(x);
                } else {
                  e.x = ex2(x.x);
                  e.y = ex2(x.y);
                }
                const float e0 = (w >> (k & 31)) & 1u ? e.x : 0.f;
                const float e1 = (w >> ((k + 1) & 31)) & 1u ? e.y : 0.f;
                acc[(i >> 1) & 1] = fadd2(acc[(i >> 1) & 1], make_float2(e0, e1));
                pk[k >> 1] = pack_bf16(e0, e1);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) pk[4 * gi + i] = 0u;
            }
          }
          return (acc[0].x + acc[0].y) + (acc[1].x + acc[1].y);
        };
        // Rows with nothing accumulated yet take the chunk's exact masked max (over both halves).
        float m_use = m_ref;
        const bool fresh = m_ref == -INFINITY;
        if (__any_sync(0xffffffffu, fresh)) {
          const float hm = half_max();
          float om;
          if (!(ok = exchange(0, hm, om))) break;
          if (fresh) m_use = fmaxf(hm, om) * c2;
        }
        float sum = exps(m_use);
        if (lane == 0) FWN_TR(26, c);
        // A half-row sum above 2^16 means some p may exceed 2^16 (the accumulators stay far from fp32
        // overflow below that): then the pair redoes the chunk exactly against the chunk's max. The flag is
        // posted now and collected after P is in TMEM.
        const uint32_t xslot = xk & 1;
        const int bad_w = __any_sync(0xffffffffu, !(sum <= 65536.f)) ? 1 : 0;  // whole warp
        if (lane == 0) xflag[xslot * 8 + half * 4 + quarter] = bad_w;
        __syncwarp();
        if (lane == 0) mbar_arrive(xbar);
        // P buffer free once the P V MMA that last read it (chunk gg-2) is complete.
        if (!(ok = mbar_wait(p_empty(sb), ((gg >> 1) & 1) ^ 1, abort_flag))) break;
        if (lane == 0) FWN_TR(29, c);
        const uint32_t pcol = trow + C::P_COL + 64 * sb + 32 * half;
        if (j0 < n_in) tmem_st32(pcol, *reinterpret_cast<const float(*)[32]>(pk));
        if (!(ok = mbar_wait(xbar, xk & 1, abort_flag))) break;
        const int bad = xflag[xslot * 8 + half * 4 + quarter] | xflag[xslot * 8 + (1 - half) * 4 + quarter];
        ++xk;
        bool grow = false;
        float corr = 1.f;
        if (bad) {
          if (lane == 0) FWN_TR(28, c);
          const float hm = half_max();
          float om;
          if (!(ok = exchange(1, hm, om))) break;
          const float m_new = fmaxf(hm, om) * c2;
          if (m_ref == -INFINITY) {
            m_ref = m_new;
          } else if (m_new > m_ref) {
            grow = true;
            corr = ex2(m_ref - m_new);
            m_ref = m_new;
            l *= corr;
          }
          sum = exps(m_ref);
          tmem_wait_st();
          if (j0 < n_in) tmem_st32(pcol, *reinterpret_cast<const float(*)[32]>(pk));
        } else {
          m_ref = m_use;
        }
        l += sum;
        if (__any_sync(0xffffffffu, grow)) {
          // O is quiescent once P V of chunk gg-1 is complete.
          if (gg > g0) {
            const uint32_t prev = gg - 1;
            if (!(ok = mbar_wait(p_empty(prev & 1), (prev >> 1) & 1, abort_flag))) break;
          }
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < D / 64; ++j) {
            float o[32];
            const uint32_t col = trow + C::O_COL + (D / 2) * half + 32 * j;
            tmem_ld32(col, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(col, o);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(sb));
        if (lane == 0) FWN_TR(21, c);
      }
      if (!ok) break;
      g = g0 + nch;
      // ---------------------------------------------------------------- epilogue
      float lo = 0.f;
      if (!(ok = exchange(2, l, lo))) break;
      const float lt = l + lo;
      const bool has = lt > 0.f;
      const float inv = has ? 1.f / lt : 0.f;
      if (half == 0 && p.lse != nullptr) {
        const float lse = has ? (m_ref + lg2(lt)) * 0.69314718055994530942f : -INFINITY;
        p.lse[static_cast<size_t>(bh) * p.lse_rows + qrow] = lse;
      }
      const bool store = qrow < p.n;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                      (static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(qrow) * p.o_sn +
                       static_cast<int64_t>(h) * p.o_sh) * C::ES + (D / 2) * C::ES * half;
      if (nch == 0) {
        if (store)
          for (int i = 0; i < D * C::ES / 32; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(0, 0, 0, 0);
        continue;
      }
      if (!(ok = mbar_wait(o_full, qc & 1, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < D / 64; ++j) {
        float o[32];
        tmem_ld32(trow + C::O_COL + (D / 2) * half + 32 * j, o);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            reinterpret_cast<uint4*>(orow + j * 64)[i] =
                make_uint4(pack_bf16(o[8 * i] * inv, o[8 * i + 1] * inv), pack_bf16(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                           pack_bf16(o[8 * i + 4] * inv, o[8 * i + 5] * inv), pack_bf16(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      ++qc;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
#undef FWN_TR
}

}  // namespace fwn
