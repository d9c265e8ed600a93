// Backward kernels for dense neighbourhoods (bf16, 128-row tile lists): 128-column chunks.
//
// Same algorithm as attn_bwd.cuh (_bwd_dq_kernel / _bwd_dkv_kernel, src/faster_weathernext/pallas_attn.py:
// 161-215): P = where(valid, exp(S - lse), 0), dS = P (dP - delta), dQ = scale dS K, dK = scale dS^T Q,
// dV = P^T dO; every output row is owned by one CTA (no atomics, deterministic).
//
// Why separate kernels: as in the forward, tcgen05.mma instructions with N = 32 or 64 leave most of the
// tensor core idle on dense masks. Here a chunk is four consecutive tiles of the list (128 columns), so
// S and dP are N = 128 MMAs and the accumulating MMAs have K = 128. Two passes ("kinds"), one CTA per SM each:
//               dQ              dK and dV
//   rows        queries         keys            (128 per work item, held all item long)
//   R0, R1      Q, dO           K, V
//   C0, C1      K, V            Q, dO           (per chunk, in rings)
//   S  = R0 C0^T, dP = R1 C1^T
//   acc += G C                  dQ += dS K; dV += P^T dO, dK += dS^T Q (C read MN-major)
// dQ: G = dS (bf16, 128 x 128) is written by the elementwise warps into TMEM and is the A operand of the
// accumulating MMA (two G buffers); K (read again by the dQ MMA) lives in a ring of three slots, V in a ring of
// two; S and dP of chunk c+1 go ahead of the dQ MMA of chunk c. dK and dV: S, dP and both accumulators take all
// 512 TMEM columns at head_dim 128, so P is written over S and dS over dP (packed bf16 pairs in the first 16
// columns of each 32-column tile); one S / dP buffer: per chunk the pipe runs dV(c), S(c+1), dK(c), dP(c+1),
// so that S of the next chunk runs while the elementwise warps compute dS; Q and dO in rings of two (three at
// head_dim 64). Rows are keys for dK / dV: the
// columns' lse and delta come with the chunk (a ring of vectors); for dQ they are per thread.
//
// Roles (576 threads): warp 0 TMA producer; warp 1 TMEM allocation and MMA issue (the warp runs the loop
// with warp-uniform descriptors, one elected lane issues); warps 2-17 elementwise, four per TMEM lane
// quadrant (thread = row), one 32-column tile of each chunk each; the mask words are read from global
// memory one chunk ahead. Epilogue: each warp stores a quarter of the accumulator columns. Every mbarrier
// wait is bounded (common.cuh).
#pragma once

#include <cuda.h>

#include "attn_bwd.cuh"
#include "common.cuh"

namespace fwn {

template <int KIND, int D>
struct BwdWideCfg {
  static_assert(KIND == kBwdDQ || KIND == kBwdDKV, "wide passes: dQ; dK and dV");
  // dK and dV in one pass (kBwdDKV): one S / dP buffer, P written over S and dS over dP (bf16 pairs, in the
  // first 16 of each 32-column tile's columns), accumulators dV and dK in the other 256 columns.
  static constexpr bool FUSED = KIND == kBwdDKV;
  static constexpr bool ROWS_ARE_KEYS = FUSED;
  static constexpr int ES = 2;
  static constexpr int EPB = 64;
  static constexpr int CB = D / EPB;
  static constexpr int ROWS = 128;
  static constexpr int SUB = 32;
  static constexpr int CH = 4;
  static constexpr int COLS = SUB * CH;
  static constexpr int NR = 2;
  static constexpr int R_BYTES = CB * ROWS * 128;
  static constexpr int C_BYTES = CB * COLS * 128;
  // C0 / C1 rings. dQ: C0 (K) is read again by the dQ MMA (three slots), C1 (V) only by dP (two). Fused: both
  // operands are read again by an accumulating MMA; chunks run one after the other (one S / dP buffer), so two
  // slots each keep the next chunk's copies in flight.
  static constexpr int N0 = FUSED ? (D == 128 ? 2 : 3) : 3;
  static constexpr int N1 = FUSED ? (D == 128 ? 2 : 3) : 2;
  static constexpr int NVEC = ROWS_ARE_KEYS ? 2 : 0;  // lse / delta vectors of the chunk's columns (1 KB)
  static constexpr int NVEC_RING = NVEC > 0 ? NVEC : 1; // ring arithmetic (no vectors for dQ)
  static constexpr int OFF_C0 = NR * R_BYTES;
  static constexpr int OFF_C1 = OFF_C0 + N0 * C_BYTES;
  static constexpr int OFF_VEC = OFF_C1 + N1 * C_BYTES;
  static constexpr int OFF_BAR = OFF_VEC + NVEC * 1024;
  static constexpr int N_BAR = 2 + 2 * N0 + 2 * N1 + 2 * NVEC + 2 + 4 + 3;
  // The dynamic shared memory base is 1024-byte aligned (checked at run time): no alignment slack.
  static constexpr int SMEM_BYTES = OFF_BAR + N_BAR * 8 + 16;
  // TMEM: S (128), dP (128), then dQ (D) and G[2] (64 each), or (fused) dV (D) and dK (D).
  static constexpr int DP_COL = 128;
  static constexpr int ACC_COL = 256;
  static constexpr int G_COL = ACC_COL + D;      // dQ
  static constexpr int ACC_K_COL = ACC_COL + D;  // fused: dK
  static constexpr int TMEM_COLS = 512;
  // Elementwise warps: four per TMEM lane quadrant, one 32-column tile of the chunk each (18 warps: at most
  // 102 registers per thread, as each sub-partition holds 16,384 and takes five warps).
  static constexpr int EW = 16;
  static constexpr int THREADS = 64 + 32 * EW;
  static constexpr int MAX_REGS = 96;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(FUSED ? ACC_K_COL + D <= TMEM_COLS : G_COL + 128 <= TMEM_COLS, "TMEM budget");
};

template <int KIND, int D>
__global__ void __maxnreg__((BwdWideCfg<KIND, D>::MAX_REGS))
    attn_bwd_wide_kernel(const __grid_constant__ CUtensorMap tm_r0, const __grid_constant__ CUtensorMap tm_r1,
                         const __grid_constant__ CUtensorMap tm_c0, const __grid_constant__ CUtensorMap tm_c1,
                         const __grid_constant__ CUtensorMap tm_c0w, const __grid_constant__ CUtensorMap tm_c1w,
                         const BwdParams p) {
  using C = BwdWideCfg<KIND, D>;
  extern __shared__ __align__(1024) uint8_t smem_bwd_wide[];
  uint8_t* smem = smem_bwd_wide;
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {
    // The tile layouts need 1024-byte aligned shared memory; report and leave (uniformly, before any wait).
    if (threadIdx.x == 0) atomicOr(&g_device_error, 0x100u);
    return;
  }
  auto r_op = [&](int i) { return sbase + i * C::R_BYTES; };
  auto c0_slot = [&](int s) { return sbase + C::OFF_C0 + s * C::C_BYTES; };
  auto c1_slot = [&](int s) { return sbase + C::OFF_C1 + s * C::C_BYTES; };
  auto vec_slot = [&](int s) { return sbase + C::OFF_VEC + s * 1024; };
  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t r_full = bar0, r_empty = bar0 + 8;
  auto c0_full = [&](int s) { return bar0 + 16 + 8 * s; };
  auto c0_empty = [&](int s) { return bar0 + 16 + 8 * (C::N0 + s); };
  const uint32_t bar1 = bar0 + 16 + 16 * C::N0;
  auto c1_full = [&](int s) { return bar1 + 8 * s; };
  auto c1_empty = [&](int s) { return bar1 + 8 * (C::N1 + s); };
  const uint32_t bar2 = bar1 + 16 * C::N1;
  auto v_full = [&](int s) { return bar2 + 8 * s; };
  auto v_empty = [&](int s) { return bar2 + 8 * (C::NVEC + s); };
  const uint32_t bar3 = bar2 + 16 * C::NVEC;
  const uint32_t s_full = bar3, s_empty = bar3 + 8;  // fused: s_empty is "dP done"
  const uint32_t bar4 = bar3 + 16;
  auto g_full = [&](int b) { return bar4 + 8 * b; };
  auto g_empty = [&](int b) { return bar4 + 16 + 8 * b; };
  const uint32_t acc_full = bar4 + 32, acc_empty = bar4 + 40, drain = bar4 + 48;
  // Fused dK / dV pass (the same slots): S and dP done (MMA commits), P and dS written (elementwise arrivals),
  // S and dP columns free again (the dV / dK MMAs that read P / dS are complete).
  [[maybe_unused]] const uint32_t f_s_full = s_full, f_dp_full = s_empty;
  [[maybe_unused]] const uint32_t f_p_full = g_full(0), f_ds_full = g_full(1), f_s_free = g_empty(0), f_dp_free = g_empty(1);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + C::N_BAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + C::N_BAR * 8 + 4);
  int trace_count = 0;  // FWN_TRACE builds: this lane's event count
#define FWN_TR(code, arg) trace_event(p.trace, trace_count, (code), (arg))

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr float kLog2e = 1.4426950408889634f;
  if (threadIdx.x == 0) {
    mbar_init(r_full, 1);
    mbar_init(r_empty, 1);
    for (int s = 0; s < C::N0; ++s) {
      mbar_init(c0_full(s), 1);
      mbar_init(c0_empty(s), 1);
    }
    for (int s = 0; s < C::N1; ++s) {
      mbar_init(c1_full(s), 1);
      mbar_init(c1_empty(s), 1);
    }
    for (int s = 0; s < C::NVEC; ++s) {
      mbar_init(v_full(s), 2);  // delta copies (expect_tx) + the producer lanes' lse stores
      mbar_init(v_empty(s), C::EW);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, C::FUSED ? 1 : C::EW);  // fused: dP done (MMA commit)
    for (int b = 0; b < 2; ++b) {
      mbar_init(g_full(b), C::EW);
      mbar_init(g_empty(b), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, C::EW);
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_r0);
    if (C::NR == 2) tma_prefetch_desc(&tm_r1);
    tma_prefetch_desc(&tm_c0);
    tma_prefetch_desc(&tm_c1);
    tma_prefetch_desc(&tm_c0w);
    tma_prefetch_desc(&tm_c1w);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int per_bh = p.np;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    uint32_t n0 = 0, n1 = 0, nvec = 0, qc = 0;  // copies issued per ring
    bool ok = true;
    int pending_r = 0;
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
      auto meta = [&](int c) { const int i = C::CH * c + (lane & 3); return i < n_sub ? __ldg(p.kb2 + t0 + i) : 0; };
      if (!(ok = mbar_wait(r_empty, (qc & 1) ^ 1, abort_flag))) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(r_full, C::NR * C::R_BYTES);
        for (int cb = 0; cb < C::CB; ++cb) {
          tma_load_4d(r_op(0) + cb * C::ROWS * 128, &tm_r0, cb * C::EPB, h, pb * C::ROWS, b, r_full);
          if (C::NR == 2) tma_load_4d(r_op(1) + cb * C::ROWS * 128, &tm_r1, cb * C::EPB, h, pb * C::ROWS, b, r_full);
        }
      }
      pending_r = 1;
      // One column operand of a chunk: one 128-row box per column block for four consecutive tiles, else one
      // 32-row box per tile and column block (lanes 0 .. n_in * CB - 1).
      auto load_op = [&](uint32_t dst, const CUtensorMap* t32, const CUtensorMap* t128, int kbl, int n_in,
                         uint32_t bar) {
        const int k0 = __shfl_sync(0xffffffffu, kbl, 0), k1 = __shfl_sync(0xffffffffu, kbl, 1);
        const int k2 = __shfl_sync(0xffffffffu, kbl, 2), k3 = __shfl_sync(0xffffffffu, kbl, 3);
        const bool run = n_in == 4 && k1 == k0 + 1 && k2 == k0 + 2 && k3 == k0 + 3;
        if (lane == 0) mbar_arrive_expect_tx(bar, n_in * C::SUB * D * C::ES);
        __syncwarp();
        if (run) {
          if (lane < C::CB) tma_load_4d(dst + lane * C::COLS * 128, t128, lane * C::EPB, h, k0 * C::SUB, b, bar);
        } else if (lane < n_in * C::CB) {
          const int s = lane / C::CB, cb = lane % C::CB;
          const int kb = s == 0 ? k0 : s == 1 ? k1 : s == 2 ? k2 : k3;
          tma_load_4d(dst + cb * C::COLS * 128 + s * C::SUB * 128, t32, cb * C::EPB, h, kb * C::SUB, b, bar);
        }
      };
      // lse and delta of the chunk's columns (rows are keys): lane s < n_in copies tile s's 32 + 32 floats.
      // delta by bulk copies (lane s < n_in: tile s); lse stored by the lanes as -lse log2 e (lane j of tile s:
      // column 32 s + j), so that the elementwise warps add it without a multiply; v_full takes both arrivals.
      auto load_vec = [&](int kbl, int n_in) -> bool {
        float nl2[C::CH];
#pragma unroll
        for (int s = 0; s < C::CH; ++s) {
          const int kb_s = __shfl_sync(0xffffffffu, kbl, s);
          nl2[s] = s < n_in ? __ldg(p.lse + static_cast<size_t>(bh) * p.lse_rows +
                                    static_cast<size_t>(kb_s) * C::SUB + lane) * -kLog2e
                            : 0.f;
        }
        if (!mbar_wait(v_empty(nvec % C::NVEC_RING), ((nvec / C::NVEC_RING) & 1) ^ 1, abort_flag)) return false;
        const int slot = nvec % C::NVEC_RING;
        const uint32_t dst = vec_slot(slot), bar = v_full(slot);
        if (lane == 0) mbar_arrive_expect_tx(bar, n_in * 128);
        __syncwarp();
        if (lane < n_in) {
          const size_t vo = static_cast<size_t>(bh) * p.lse_rows + static_cast<size_t>(kbl) * C::SUB;
          bulk_load(dst + 512 + lane * 128, p.delta + vo, 128, bar);
        }
        float* vl = reinterpret_cast<float*>(smem + C::OFF_VEC + slot * 1024);
#pragma unroll
        for (int s = 0; s < C::CH; ++s)
          if (s < n_in) vl[32 * s + lane] = nl2[s];
        __syncwarp();
        if (lane == 0) mbar_arrive(bar);  // second arrival: publishes the lanes' stores
        ++nvec;
        return true;
      };
      int kb_cur = meta(0);
      for (int c = 0; c < nch && ok; ++c) {
        const int kb_next = c + 1 < nch ? meta(c + 1) : 0;
        const int n_in = min(C::CH, n_sub - C::CH * c);
        if (!(ok = mbar_wait(c0_empty(n0 % C::N0), ((n0 / C::N0) & 1) ^ 1, abort_flag))) break;
        if (lane == 0) FWN_TR(3, c);
        load_op(c0_slot(n0 % C::N0), &tm_c0, &tm_c0w, kb_cur, n_in, c0_full(n0 % C::N0));
        ++n0;
        if (!(ok = mbar_wait(c1_empty(n1 % C::N1), ((n1 / C::N1) & 1) ^ 1, abort_flag))) break;
        load_op(c1_slot(n1 % C::N1), &tm_c1, &tm_c1w, kb_cur, n_in, c1_full(n1 % C::N1));
        ++n1;
        if constexpr (C::ROWS_ARE_KEYS) {
          if (!(ok = load_vec(kb_cur, n_in))) break;
        }
        kb_cur = kb_next;
      }
      if (!ok) break;
      ++qc;
    }
    if (!ok && lane == 0) {
      volatile int never = 0;
      for (uint32_t k = (n0 >= C::N0 ? n0 - C::N0 : 0); k < n0; ++k) mbar_wait(c0_full(k % C::N0), (k / C::N0) & 1, &never);
      for (uint32_t k = (n1 >= C::N1 ? n1 - C::N1 : 0); k < n1; ++k) mbar_wait(c1_full(k % C::N1), (k / C::N1) & 1, &never);
      if (C::NVEC)
        for (uint32_t k = (nvec >= C::NVEC_RING ? nvec - C::NVEC_RING : 0); k < nvec; ++k)
          mbar_wait(v_full(k % C::NVEC_RING), (k / C::NVEC_RING) & 1, &never);
      if (pending_r) mbar_wait(r_full, qc & 1, &never);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (whole warp, one lane issues)
    constexpr uint32_t kIdescAcc = instr_desc(false, 128, D, false, true);
    const uint64_t r0desc = smem_desc(r_op(0), 16, 1024), r1desc = smem_desc(r_op(1), 16, 1024);
    uint32_t g = 0, qc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh;
      const int t0 = p.ptr2[pb], n_sub = p.ptr2[pb + 1] - t0;
      const int nch = (n_sub + C::CH - 1) / C::CH;
      if (nch == 0) continue;
      if (!(ok = warp_wait(r_full, qc & 1, abort_flag))) break;
      const uint32_t g0 = g;
      if constexpr (C::FUSED) {
        // On the tensor pipe per chunk c: dV(c) once P(c) is written; S(c+1) over P(c) once dV(c) is complete
        // (MMAs into different accumulators are not ordered, so the warp waits for dV's commit); dK(c) once dS(c)
        // is written; dP(c+1) over dS(c) once dK(c) is complete. S(c+1) thus runs while the elementwise warps
        // compute dS(c), and P(c+1) can start as soon as they are done.
        auto issue_s = [&](int c) -> bool {  // S = K Q^T of chunk c (columns 0-127)
          const uint32_t gg = g0 + c;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (!warp_wait(c0_full(gg % C::N0), (gg / C::N0) & 1, abort_flag)) return false;
          if (!warp_wait(f_s_free, (gg & 1) ^ 1, abort_flag)) return false;  // dV of chunk gg-1 complete
          if (lane == 0) FWN_TR(13, c);
          tc_fence_after();
          const uint32_t idesc = instr_desc(false, 128, 32 * n_in, false, false);
          const uint64_t c0desc = smem_desc(c0_slot(gg % C::N0), 16, 1024);
          if (elect_one_sync()) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t cb = kk / 4, within = (kk % 4) * 32;
              mma_ss<false>(tmem, r0desc + ((cb * C::ROWS * 128 + within) >> 4),
                            c0desc + ((cb * C::COLS * 128 + within) >> 4), idesc, kk > 0 ? 1u : 0u);
            }
            mma_commit(f_s_full);
          }
          __syncwarp();
          return true;
        };
        auto issue_dp = [&](int c) -> bool {  // dP = V dO^T of chunk c (columns 128-255)
          const uint32_t gg = g0 + c;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (!warp_wait(c1_full(gg % C::N1), (gg / C::N1) & 1, abort_flag)) return false;
          if (!warp_wait(f_dp_free, (gg & 1) ^ 1, abort_flag)) return false;  // dK of chunk gg-1 complete
          if (lane == 0) FWN_TR(17, c);
          tc_fence_after();
          const uint32_t idesc = instr_desc(false, 128, 32 * n_in, false, false);
          const uint64_t c1desc = smem_desc(c1_slot(gg % C::N1), 16, 1024);
          if (elect_one_sync()) {
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t cb = kk / 4, within = (kk % 4) * 32;
              mma_ss<false>(tmem + C::DP_COL, r1desc + ((cb * C::ROWS * 128 + within) >> 4),
                            c1desc + ((cb * C::COLS * 128 + within) >> 4), idesc, kk > 0 ? 1u : 0u);
            }
            mma_commit(f_dp_full);
            // S of every chunk of the item is issued before its last dP: the rows are free once this completes.
            if (c == nch - 1) mma_commit(r_empty);
          }
          __syncwarp();
          if (lane == 0) FWN_TR(11, c);
          return true;
        };
        ok = issue_s(0) && issue_dp(0);
        for (int c = 0; c < nch && ok; ++c) {
          const uint32_t gg = g0 + c;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          const int s0 = gg % C::N0, s1 = gg % C::N1;
          // A = P / dS from TMEM: K-step kk reads 8 columns of packed pairs at 32 (kk / 2) + 8 (kk % 2).
          const int ksteps = 2 * n_in;
          if (!(ok = warp_wait(f_p_full, gg & 1, abort_flag))) break;
          if (c == 0 && !(ok = warp_wait(acc_empty, (qc & 1) ^ 1, abort_flag))) break;
          if (lane == 0) FWN_TR(15, c);
          tc_fence_after();
          if (elect_one_sync()) {
            const uint64_t bdesc = smem_desc(c1_slot(s1), C::COLS * 128, 1024);
            for (int kk = 0; kk < ksteps; ++kk)
              mma_ts(tmem + C::ACC_COL, tmem + 32 * (kk >> 1) + 8 * (kk & 1), bdesc + ((kk * 16 * 128) >> 4),
                     kIdescAcc, (c == 0 && kk == 0) ? 0u : 1u);
            mma_commit(f_s_free);
            mma_commit(c1_empty(s1));
          }
          __syncwarp();
          if (c + 1 < nch && !(ok = issue_s(c + 1))) break;
          if (!(ok = warp_wait(f_ds_full, gg & 1, abort_flag))) break;
          if (lane == 0) FWN_TR(16, c);
          tc_fence_after();
          if (elect_one_sync()) {
            const uint64_t bdesc = smem_desc(c0_slot(s0), C::COLS * 128, 1024);
            for (int kk = 0; kk < ksteps; ++kk)
              mma_ts(tmem + C::ACC_K_COL, tmem + C::DP_COL + 32 * (kk >> 1) + 8 * (kk & 1),
                     bdesc + ((kk * 16 * 128) >> 4), kIdescAcc, (c == 0 && kk == 0) ? 0u : 1u);
            mma_commit(f_dp_free);
            mma_commit(c0_empty(s0));
            if (c == nch - 1) mma_commit(acc_full);
          }
          __syncwarp();
          if (lane == 0) FWN_TR(12, c);
          if (c + 1 < nch && !(ok = issue_dp(c + 1))) break;
        }
      } else {
        // dQ: S and dP of chunk c+1 ahead of the dQ MMA of chunk c (which reads dS from one of two G buffers).
        for (int c = 0; c <= nch && ok; ++c) {
          if (c < nch) {
            const uint32_t gg = g0 + c;
            const int n_in = min(C::CH, n_sub - C::CH * c);
            if (!(ok = warp_wait(c0_full(gg % C::N0), (gg / C::N0) & 1, abort_flag))) break;
            if (!(ok = warp_wait(c1_full(gg % C::N1), (gg / C::N1) & 1, abort_flag))) break;
            if (!(ok = warp_wait(s_empty, (gg & 1) ^ 1, abort_flag))) break;
            if (lane == 0) FWN_TR(13, c);
            tc_fence_after();
            const uint32_t idesc = instr_desc(false, 128, 32 * n_in, false, false);
            const uint64_t c0desc = smem_desc(c0_slot(gg % C::N0), 16, 1024);
            const uint64_t c1desc = smem_desc(c1_slot(gg % C::N1), 16, 1024);
            if (elect_one_sync()) {
  #pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t cb = kk / 4, within = (kk % 4) * 32;
                mma_ss<false>(tmem, r0desc + ((cb * C::ROWS * 128 + within) >> 4),
                              c0desc + ((cb * C::COLS * 128 + within) >> 4), idesc, kk > 0 ? 1u : 0u);
              }
  #pragma unroll
              for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t cb = kk / 4, within = (kk % 4) * 32;
                mma_ss<false>(tmem + C::DP_COL, r1desc + ((cb * C::ROWS * 128 + within) >> 4),
                              c1desc + ((cb * C::COLS * 128 + within) >> 4), idesc, kk > 0 ? 1u : 0u);
              }
              mma_commit(c1_empty(gg % C::N1));  // C1 (V) is read only by dP
              mma_commit(s_full);
              if (c == nch - 1) mma_commit(r_empty);
            }
            __syncwarp();
            if (lane == 0) FWN_TR(11, c);
          }
          if (c >= 1) {
            const uint32_t gg = g0 + c - 1;
            const int gb = gg & 1;
            const int n_in = min(C::CH, n_sub - C::CH * (c - 1));
            if (!(ok = warp_wait(g_full(gb), (gg >> 1) & 1, abort_flag))) break;
            if (c == 1 && !(ok = warp_wait(acc_empty, (qc & 1) ^ 1, abort_flag))) break;
            if (lane == 0) FWN_TR(14, c - 1);
            tc_fence_after();
            const uint64_t bdesc = smem_desc(c0_slot(gg % C::N0), C::COLS * 128, 1024);
            const uint32_t gcol = tmem + C::G_COL + 64 * gb;
            const int ksteps = 2 * n_in;
            if (elect_one_sync()) {
              for (int kk = 0; kk < ksteps; ++kk)
                mma_ts(tmem + C::ACC_COL, gcol + 8 * kk, bdesc + ((kk * 16 * 128) >> 4), kIdescAcc,
                       (c == 1 && kk == 0) ? 0u : 1u);
              mma_commit(g_empty(gb));
              mma_commit(c0_empty(gg % C::N0));
              if (c == nch) mma_commit(acc_full);
            }
            __syncwarp();
            if (lane == 0) FWN_TR(12, c - 1);
          }
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
    // ------------------------------------------------------------------ elementwise + epilogue (warps 2-17)
    // Warp w: TMEM lane quadrant w % 4 (thread = row), tile j = (w - 2) / 4 of each chunk (32 columns).
    const int quarter = warp & 3, j = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    const float c2 = p.scale_log2;
    uint32_t g = 0, qc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh, bh = it / per_bh, h = bh % p.heads, b = bh / p.heads;
      const int t0 = p.ptr2[pb], n_sub = p.ptr2[pb + 1] - t0;
      const int nch = (n_sub + C::CH - 1) / C::CH;
      const int grow = pb * C::ROWS + row;
      float nl2_row = 0.f, delta_row = 0.f;
      if (!C::ROWS_ARE_KEYS) {
        nl2_row = -p.lse[static_cast<size_t>(bh) * p.lse_rows + grow] * kLog2e;
        delta_row = p.delta[static_cast<size_t>(bh) * p.lse_rows + grow];
      }
      // Mask word of this warp's tile of chunk c (global memory, read one chunk ahead).
      auto word = [&](int c) -> uint32_t {
        const int i = C::CH * c + j;
        return i < n_sub ? __ldg(p.bits2 + static_cast<size_t>(t0 + i) * 128 + row) : 0u;
      };
      uint32_t nw = nch > 0 ? word(0) : 0u;
      const uint32_t g0 = g;
      if constexpr (C::FUSED) {
        for (int c = 0; c < nch; ++c) {
          const uint32_t gg = g0 + c;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          const uint32_t w = nw;
          if (c + 1 < nch) nw = word(c + 1);
          const uint32_t a = __reduce_or_sync(0xffffffffu, w);
          const uint32_t vs = gg % C::NVEC_RING;
          if (!(ok = mbar_wait(v_full(vs), (gg / C::NVEC_RING) & 1, abort_flag))) break;
          const uint32_t vslot = vec_slot(vs) + 128 * j;
          if (!(ok = mbar_wait(f_s_full, gg & 1, abort_flag))) break;
          if (lane == 0) FWN_TR(20, c);
          tc_fence_after();
          // P = exp2(S scale log2 e - lse log2 e) on the allowed columns, kept in s (fp32) for dS and written
          // as packed bf16 pairs over this tile's own S columns (read above by this warp only).
          float s[32];
          if (j < n_in) tmem_ld32(trow + 32 * j, s);
          tmem_wait_ld();
          uint32_t pk[16];
          const float2 cc = make_float2(c2, c2);
#pragma unroll
          for (int gi = 0; gi < 4; ++gi) {
            if ((a >> (8 * gi)) & 0xFFu) {
              const uint32_t va = vslot + 32 * gi;
              const float4 l0 = ld_shared_f32x4(va), l1 = ld_shared_f32x4(va + 16);
              const float lv[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};  // -lse log2 e
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const int k = 8 * gi + i;
                const float2 x = ffma2(make_float2(s[k], s[k + 1]), cc, make_float2(lv[i], lv[i + 1]));
                // MUFU.EX2 for every column: the backward is not bound by that pipe, and moving a quarter of the
                // exponentials to the FMA-pipe polynomial (as the forward does) made dK/dV and dQ 2-3 % slower.
                const float2 e = make_float2(ex2(x.x), ex2(x.y));
                s[k] = (w >> k) & 1u ? e.x : 0.f;
                s[k + 1] = (w >> (k + 1)) & 1u ? e.y : 0.f;
                pk[k >> 1] = pack_bf16(s[k], s[k + 1]);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) pk[4 * gi + i] = 0u;
            }
          }
          if (j < n_in) tmem_st16(trow + 32 * j, pk);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(f_p_full);
          if (lane == 0) FWN_TR(22, c);
          // dS = P (dP - delta), over this tile's dP columns.
          if (!(ok = mbar_wait(f_dp_full, gg & 1, abort_flag))) break;
          if (lane == 0) FWN_TR(23, c);
          tc_fence_after();
          // dP in two halves of 16 columns while P stays in s (fp32): a thread holds 48 values instead of 64, which the
          // 96-register budget of 18 warps keeps without spilling (dK/dV about 1 % faster at the WN2 shape).
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float dp[16];
            if (j < n_in) tmem_ld16(trow + C::DP_COL + 32 * j + 16 * hf, dp);
            tmem_wait_ld();
#pragma unroll
            for (int g2 = 0; g2 < 2; ++g2) {
              const int gi = 2 * hf + g2;
              if ((a >> (8 * gi)) & 0xFFu) {
                const uint32_t va = vslot + 512 + 32 * gi;
                const float4 d0 = ld_shared_f32x4(va), d1 = ld_shared_f32x4(va + 16);
                const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
                for (int i = 0; i < 8; i += 2) {
                  const int k = 8 * gi + i, kk = 8 * g2 + i;
                  const float2 ds = fmul2(make_float2(s[k], s[k + 1]),
                                          fsub2(make_float2(dp[kk], dp[kk + 1]), make_float2(dv[i], dv[i + 1])));
                  pk[k >> 1] = pack_bf16(ds.x, ds.y);
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(v_empty(vs));
          if (j < n_in) tmem_st16(trow + C::DP_COL + 32 * j, pk);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(f_ds_full);
          if (lane == 0) FWN_TR(21, c);
        }
      } else {
        // dQ: rows are queries (lse and delta per thread); dS = P (dP - delta) into G buffer gg & 1.
        for (int c = 0; c < nch; ++c) {
          const uint32_t gg = g0 + c;
          const int gb = gg & 1;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          const uint32_t w = nw;
          if (c + 1 < nch) nw = word(c + 1);
          const uint32_t a = __reduce_or_sync(0xffffffffu, w);
          if (!(ok = mbar_wait(s_full, gg & 1, abort_flag))) break;
          if (lane == 0) FWN_TR(20, c);
          tc_fence_after();
          // S and dP of this tile -> registers; then the buffer is released for the next S / dP MMAs.
          float s[32], dp[32];
          if (j < n_in) {
            tmem_ld32(trow + 32 * j, s);
            tmem_ld32(trow + C::DP_COL + 32 * j, dp);
          }
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(s_empty);
          uint32_t pk[16];
          const float2 cc = make_float2(c2, c2), nl2 = make_float2(nl2_row, nl2_row);
          const float2 dl = make_float2(delta_row, delta_row);
#pragma unroll
          for (int gi = 0; gi < 4; ++gi) {
            if ((a >> (8 * gi)) & 0xFFu) {
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const int k = 8 * gi + i;
                const float2 x = ffma2(make_float2(s[k], s[k + 1]), cc, nl2);
                float2 e = make_float2(ex2(x.x), ex2(x.y));  // MUFU.EX2 for every column (see the fused pass)
                e.x = (w >> k) & 1u ? e.x : 0.f;
                e.y = (w >> (k + 1)) & 1u ? e.y : 0.f;
                const float2 ds = fmul2(e, fsub2(make_float2(dp[k], dp[k + 1]), dl));
                pk[k >> 1] = pack_bf16(ds.x, ds.y);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) pk[4 * gi + i] = 0u;
            }
          }
          if (lane == 0) FWN_TR(26, c);
          // G buffer free once the dQ MMA of chunk gg-2 is complete.
          if (!(ok = mbar_wait(g_empty(gb), ((gg >> 1) & 1) ^ 1, abort_flag))) break;
          if (j < n_in) tmem_st16(trow + C::G_COL + 64 * gb + 16 * j, pk);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(g_full(gb));
          if (lane == 0) FWN_TR(21, c);
        }
      }
      if (!ok) break;
      g = g0 + nch;
      // ---------------------------------------------------------------- epilogue: this warp's D / 4 columns
      constexpr int OC = D / 4;
      const bool store = grow < p.n;
      const int64_t roff = (static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(grow) * p.o_sn +
                            static_cast<int64_t>(h) * p.o_sh) * C::ES + OC * C::ES * j;
      // Accumulators: dK (scaled, to out0) and / or dV (to out1); fused passes store both.
      constexpr int NACC = C::FUSED ? 2 : 1;
      if (nch == 0) {
        if (store)
          for (int ai = 0; ai < NACC; ++ai) {
            uint8_t* dst = reinterpret_cast<uint8_t*>((!C::FUSED || ai == 1) ? p.out0 : p.out1) + roff;
            for (int i = 0; i < OC * C::ES / 16; ++i) reinterpret_cast<uint4*>(dst)[i] = make_uint4(0, 0, 0, 0);
          }
        continue;
      }
      if (!(ok = mbar_wait(acc_full, qc & 1, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int ai = 0; ai < NACC; ++ai) {
        const bool is_dk = !C::FUSED || ai == 1;  // dQ or (fused) dK: scaled, to out0
        uint8_t* dst = reinterpret_cast<uint8_t*>(is_dk ? p.out0 : p.out1) + roff;
        const float mul = is_dk ? p.scale : 1.f;
        const uint32_t acc_col = C::FUSED && ai == 1 ? C::ACC_K_COL : C::ACC_COL;
#pragma unroll
        for (int jj = 0; jj < OC / 16; ++jj) {
          float o[16];
          tmem_ld16(trow + acc_col + OC * j + 16 * jj, o);
          tmem_wait_ld();
          if (store) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
              reinterpret_cast<uint4*>(dst + jj * 32)[i] =
                  make_uint4(pack_bf16(o[8 * i] * mul, o[8 * i + 1] * mul), pack_bf16(o[8 * i + 2] * mul, o[8 * i + 3] * mul),
                             pack_bf16(o[8 * i + 4] * mul, o[8 * i + 5] * mul), pack_bf16(o[8 * i + 6] * mul, o[8 * i + 7] * mul));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty);
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
