// Forward kernel of the block-sparse masked flash attention (sm_100a, tcgen05 + TMA).
//
// Replaces the Pallas-Triton `_kernel` (src/faster_weathernext/pallas_attn.py:112-141). Same math:
// per query row, an online softmax over the allowed keys of the row's query block's active 32-key
// tiles; masked logits contribute exactly 0 (the reference sets them to -1e30 so exp underflows to
// 0, pallas_attn.py:123-125); O = acc / l; LSE = m + log(l).
//
// Work item = (batch, head, 128-query block of the paired tile list). Persistent CTAs walk items
// blockIdx.x, +gridDim.x, ... Roles (192 threads):
//   warp 0      TMA producer: Q tile once per item; per chunk of up to two 32-key tiles, the K and V
//               tiles and the tiles' mask words. Tile mode: 32 consecutive keys per tile (4D tensor
//               maps over [B, n, H, D], 128-byte swizzle). Gathered mode: the 32 keys of a tile are the
//               block's distinct keys in ascending order (cols), fetched 4 rows at a time with TMA
//               tile::gather4 from a 2D view of K / V; the swizzle is by shared-memory address, so
//               8 gathers at 512-byte steps build the same 32-row tile.
//   warp 1      TMEM allocation; one thread issues the tcgen05 MMAs:
//                 S[buf] = Q K^T  (M=128, N=32|64, K=D)        -> TMEM, fp32
//                 O     += P V    (M=128, N=D,     K=32|64)     -> TMEM, fp32 (P from TMEM for bf16,
//                                                                          from shared memory for tf32)
//               S of chunk c+1 is issued before P V of chunk c, so the tensor core overlaps softmax.
//   warps 2-5   softmax: thread = query row = TMEM lane. Reads S with tcgen05.ld, applies the row's
//               mask word, keeps a running max m (log2 domain) and sum l, writes P (bf16 to TMEM,
//               fp32 to shared memory) for the P V MMA. O is rescaled in TMEM only when the row max grows by
//               more than 2^8 (the final O / l is exact either way). Exponentials are issued only for
//               columns that some row of the warp may attend to.
//               Epilogue: O / l -> global, LSE -> global.
// Every mbarrier wait is bounded (common.cuh); on expiry the CTA drains and returns with the device
// error word set.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fwn {

struct FwdParams {
  const int32_t* ptr2;    // [NP + 1] 128-row list
  const int32_t* kb2;     // [T2] key block of each tile (tile mode)
  const int32_t* cols;    // [T2 * 32] key of each slot (gathered mode)
  const uint32_t* bits2;  // [T2 * 128]
  int head_major;         // gathered mode: rows of the 2D K/V view are (b, h, node) instead of (b, node, h)
  void* o;                // [B, n, H, D]
  float* lse;             // [B, H, lse_rows] or null
  int64_t o_sb, o_sn, o_sh;
  int batch, heads, n, np, lse_rows, n_items;
  float scale_log2;       // scale * log2(e)
  unsigned long long* trace;  // FWN_TRACE builds: kTraceCtas x kTraceEvents event records (else unused)
  const void* q;          // Q and its element strides (read by the softmax warps where Q lives in TMEM)
  int64_t q_sb, q_sn, q_sh;
  unsigned long long wait_limit_ns;  // bound of every mbarrier wait of the narrow kernel (kWaitLimitNs normally)
  int fault_skip_kv;      // test launches only: the producer leaves out the first K/V load of CTA 0, so that the
                          // MMA warp's bounded wait on it expires (nothing else is changed)
};

template <int D, bool F32, bool X3 = false>
struct FwdCfg {
  static constexpr int ES = F32 ? 4 : 2;
  static constexpr int EPB = 128 / ES;        // elements per 128-byte column block
  static constexpr int CB = D / EPB;          // column blocks of a head_dim row
  static constexpr int ROWS = 128;            // query rows per item
  static constexpr int SUB = 32;              // keys per tile
  // Tiles per chunk: one at head_dim 128 (bf16: keeps two CTAs per SM, so that one CTA's softmax overlaps the
  // other's MMAs; tf32: two tiles would leave room for two K/V stages instead of four, measured 11 % slower at the
  // WN2 shape) and in 3xTF32 (operand copies); else two.
  // bf16 head_dim 64 (the sparse configurations) runs four CTAs per SM with one 32-key tile per chunk and P written
  // over S in TMEM (QUAD); the other bf16 / tf32 variants two CTAs or one.
  static constexpr bool QUAD = !F32 && D == 64;
  static constexpr int CH = (QUAD || X3 || D == 128) ? 1 : 2;
  static constexpr int KEYS = SUB * CH;       // keys per chunk
  static constexpr int KSTEP = F32 ? 8 : 16;  // K of one MMA instruction
  static constexpr int Q_BYTES = CB * ROWS * 128;
  static constexpr int KV_BYTES = CB * KEYS * 128;
  // Stage: K, V, (3xTF32: K_lo, V_lo), mask words.
  static constexpr int BITS_OFF = (X3 ? 4 : 2) * KV_BYTES;
  static constexpr int STAGE_BYTES = (BITS_OFF + CH * 512 + 1023) / 1024 * 1024;
  // bf16 and tf32: P goes to TMEM (packed bf16 pairs or fp32, the A operand of P V read from tensor memory);
  // 3xTF32 keeps P (hi and lo copies) in shared memory (128-byte swizzle).
  static constexpr bool P_TMEM = !X3;
  static constexpr int PCB = KEYS * ES / 128;  // 128-byte column blocks of a shared-memory P row
  static constexpr int P_BYTES = P_TMEM ? 0 : PCB * ROWS * 128;
  static constexpr int PBUF_BYTES = P_BYTES * (X3 ? 2 : 1);  // P (3xTF32: P_hi, P_lo)
  // tf32 (one CTA per SM): Q lives in TMEM, one fp32 element per column (the A operand of S, loaded by the softmax
  // warps: thread = row = lane), and shared memory holds only K / V stages; MMAs that take A from TMEM read a
  // quarter of the shared-memory bytes.
  static constexpr bool Q_TMEM = F32;
  static constexpr int OFF_STAGE = Q_TMEM ? 0 : Q_BYTES;
  // Bytes past the stages: P buffers, mbarriers (14 + 3 per stage), TMEM holder / abort word, 1 KB of slack to
  // align the dynamic shared memory base up to 1024 bytes.
  static constexpr int smem_bytes(int ns) { return OFF_STAGE + ns * STAGE_BYTES + 2 * PBUF_BYTES + (14 + 3 * ns) * 8 + 16 + 1024; }
  static constexpr bool fit(int ns) { return smem_bytes(ns) <= (F32 ? 227 * 1024 : QUAD ? 227 * 1024 / 4 : 227 * 1024 / 2); }
  // K/V stages: as many as fit (bf16: two CTAs per SM; tf32: one) up to 6, so that the copies of the next chunks
  // are in flight while the softmax works; 3xTF32 2.
  static constexpr int NS = fit(6) ? 6 : fit(5) ? 5 : fit(4) ? 4 : fit(3) ? 3 : 2;
  static constexpr int OFF_P = OFF_STAGE + NS * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_P + 2 * PBUF_BYTES;
  static constexpr int N_BAR = 2 + 2 * NS + 2 + 2 + 2 + 2 + 2 + 1 + 1 + NS;
  static constexpr int SMEM_BYTES = OFF_BAR + N_BAR * 8 + 16 + 1024;  // + tmem holder / abort word + slack
  // TMEM: S buffers at 0 and S_STRIDE; O at O_COL. QUAD: two 32-column S buffers, P (packed bf16 pairs) written over
  // the S it was computed from, O at 64: 128 columns, four CTAs per SM.
  static constexpr bool P_OVER_S = QUAD;
  static constexpr int S_STRIDE = QUAD ? 32 : 64;
  static constexpr int O_COL = QUAD ? 64 : 128;
  // TMEM P buffers: KEYS / 2 columns (bf16 pairs) or KEYS (tf32). One 32-key tile per chunk: in the unused upper
  // half of each 64-column S buffer; two: after O (tf32 head_dim 64 then needs 512 columns, one CTA per SM).
  static constexpr int PW = F32 ? KEYS : KEYS / 2;
  static constexpr int P_COL = P_OVER_S ? 0 : CH == 1 ? 32 : O_COL + D;
  static constexpr int P_STRIDE = P_OVER_S ? S_STRIDE : CH == 1 ? 64 : PW;
  static constexpr int Q_COL = CH == 1 ? O_COL + D : P_COL + 2 * PW;  // TMEM Q (tf32)
  static constexpr int TMEM_COLS = QUAD ? 128 : Q_TMEM ? 512 : (CH == 1 || P_COL + 2 * PW <= 256) ? 256 : 512;
  static constexpr int THREADS = X3 ? 320 : 192;  // 3xTF32: + a warpgroup splitting tiles into hi / lo
  static constexpr int MIN_BLOCKS = QUAD ? 4 : (2 * SMEM_BYTES <= 227 * 1024) ? 2 : 1;
  // Registers are allocated per warp in units of 256: 168 per thread is the most that lets two
  // 192-thread CTAs share an SM's 65,536.
  // Each SM sub-partition has 16,384 registers and takes a quarter of the resident warps (rounded up):
  // twelve warps (two CTAs) or ten (3xTF32) leave 168 per thread.
  // Four 192-thread CTAs (24 warps, six per sub-partition) leave 85: 80 in units of 8.
  static constexpr int MAX_REGS = QUAD ? 80 : (MIN_BLOCKS == 2 || X3) ? 168 : 200;
  static_assert(STAGE_BYTES % 1024 == 0 && Q_BYTES % 1024 == 0 && P_BYTES % 1024 == 0, "1 KB alignment");
  static_assert(N_BAR == 14 + 3 * NS && SMEM_BYTES == smem_bytes(NS), "shared memory layout");
  static_assert(!P_TMEM || (P_COL + P_STRIDE + PW <= TMEM_COLS && (CH == 1 || P_COL >= O_COL + D)), "TMEM budget");
  static_assert(TMEM_COLS * MIN_BLOCKS <= 512, "TMEM columns of the CTAs of an SM");
  static_assert(!QUAD || (O_COL >= 2 * S_STRIDE && O_COL + D <= TMEM_COLS && MIN_BLOCKS * SMEM_BYTES <= 227 * 1024),
                "QUAD layout");
  static_assert(!Q_TMEM || Q_COL + D * (X3 ? 2 : 1) <= TMEM_COLS, "TMEM budget (Q)");
  static_assert(D % EPB == 0, "head_dim must fill whole 128-byte column blocks");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(!X3 || F32, "3xTF32 takes float32 operands");
};

template <int D, bool F32, bool GATHER, bool X3 = false>
__global__ void __launch_bounds__(FwdCfg<D, F32, X3>::THREADS) __maxnreg__((FwdCfg<D, F32, X3>::MAX_REGS))
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_k32,
                    const __grid_constant__ CUtensorMap tm_v32, const FwdParams p) {
  using C = FwdCfg<D, F32, X3>;
  extern __shared__ uint8_t smem_fwd[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_fwd) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t q_smem = sbase;
  auto stage_k = [&](int s) { return sbase + C::OFF_STAGE + s * C::STAGE_BYTES; };
  auto stage_v = [&](int s) { return sbase + C::OFF_STAGE + s * C::STAGE_BYTES + C::KV_BYTES; };
  auto stage_bits = [&](int s) { return sbase + C::OFF_STAGE + s * C::STAGE_BYTES + C::BITS_OFF; };
  auto p_smem = [&](int b) { return sbase + C::OFF_P + b * C::PBUF_BYTES; };
  // 3xTF32 lo copies (same byte layout as their hi tiles).
  const uint32_t q_lo = sbase + C::Q_BYTES;
  auto stage_klo = [&](int s) { return sbase + C::OFF_STAGE + s * C::STAGE_BYTES + 2 * C::KV_BYTES; };
  auto stage_vlo = [&](int s) { return sbase + C::OFF_STAGE + s * C::STAGE_BYTES + 3 * C::KV_BYTES; };
  auto p_lo = [&](int b) { return sbase + C::OFF_P + b * C::PBUF_BYTES + C::P_BYTES; };
  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t q_full = bar0, q_empty = bar0 + 8;
  auto kv_full = [&](int s) { return bar0 + 16 + 8 * s; };
  auto kv_empty = [&](int s) { return bar0 + 16 + 8 * (C::NS + s); };
  const uint32_t bar1 = bar0 + 16 + 16 * C::NS;
  auto s_full = [&](int b) { return bar1 + 8 * b; };
  auto s_empty = [&](int b) { return bar1 + 16 + 8 * b; };
  auto p_full = [&](int b) { return bar1 + 32 + 8 * b; };
  auto p_empty = [&](int b) { return bar1 + 48 + 8 * b; };
  const uint32_t o_full = bar1 + 64, o_empty = bar1 + 72, drain = bar1 + 80;
  // 3xTF32: the converter's "split done" barriers; the MMA waits on these instead of the TMA ones.
  const uint32_t q_ready = bar1 + 88;
  auto kv_ready = [&](int s) { return bar1 + 96 + 8 * s; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + C::N_BAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + C::N_BAR * 8 + 4);
  const unsigned long long wlim = p.wait_limit_ns;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int trace_count = 0;  // FWN_TRACE builds: this lane's event count
#define FWN_TR(code, arg) trace_event(p.trace, trace_count, (code), (arg))
  if (threadIdx.x == 0) {
    mbar_init(q_full, C::Q_TMEM ? 4 : 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(s_empty(b), 4);
      mbar_init(p_full(b), 4);
      mbar_init(p_empty(b), 1);
    }
    mbar_init(o_full, 1);
    mbar_init(o_empty, 4);
    mbar_init(drain, 1);
    mbar_init(q_ready, 4);
    for (int st = 0; st < C::NS; ++st) mbar_init(kv_ready(st), 4);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    if (GATHER) {
      tma_prefetch_desc(&tm_k32);
      tma_prefetch_desc(&tm_v32);
    }
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  const int per_bh = p.np;
  allow_dependents();  // the delta pass may be scheduled now; it waits for this grid before reading o
  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    // Tile metadata is prefetched two chunks ahead, and the next item's list range one item ahead.
    uint32_t g = 0, qc = 0;
    bool ok = true;
    int pending_q = 0;
    long long skipped = -1;  // fault_skip_kv launches: the stage load left out
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
      ChunkMeta<C::CH> m0 = load_chunk_meta<C::CH, GATHER>(p.kb2, p.cols, t0, n_sub, 0, lane);
      ChunkMeta<C::CH> m1 = load_chunk_meta<C::CH, GATHER>(p.kb2, p.cols, t0, n_sub, 1, lane);
      if (lane == 0) FWN_TR(1, it);
      if constexpr (!C::Q_TMEM) {
        if (!(ok = mbar_wait(q_empty, (qc & 1) ^ 1, abort_flag, wlim))) break;
        if (lane == 0) {
          FWN_TR(2, nch);
          mbar_arrive_expect_tx(q_full, C::Q_BYTES);
          for (int cb = 0; cb < C::CB; ++cb)
            tma_load_4d(q_smem + cb * C::ROWS * 128, &tm_q, cb * C::EPB, h, pb * C::ROWS, b, q_full);
        }
        pending_q = 1;
      }
      // Gathered mode: row of the 2D view of K / V holding (batch b, node `key`, head h).
      const int row_base = p.head_major ? (b * p.heads + h) * p.n : b * p.n * p.heads + h;
      const int row_mul = p.head_major ? 1 : p.heads;
      // Chunk c's copies; `meta` was loaded two chunks earlier. The loop below is unrolled by two so that
      // each prefetched register pair is consumed in place (a register move would wait for the load).
      auto issue_chunk = [&](int c, const ChunkMeta<C::CH>& meta) -> bool {
          const int st = g % C::NS;
          if (!mbar_wait(kv_empty(st), ((g / C::NS) & 1) ^ 1, abort_flag, wlim)) return false;
          if (p.fault_skip_kv && it == 0 && c == 0) {
            skipped = g;  // neither the expected bytes nor any copy: kv_full of this stage never completes
            return true;
          }
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (lane == 0) FWN_TR(3, c);
          if (lane == 0) mbar_arrive_expect_tx(kv_full(st), n_in * (2 * C::SUB * D * C::ES + 512));
          __syncwarp();
  #pragma unroll
          for (int s = 0; s < C::CH; ++s) {
            if (s >= n_in) break;
            const int t = t0 + C::CH * c + s;
            if (GATHER && __all_sync(0xffffffffu, meta.v[s] == __shfl_sync(0xffffffffu, meta.v[s], 0) + lane)) {
              // The tile's 32 keys are consecutive (about 40 % of the gathered tiles at configuration 3): one
              // 32-row box per operand and column block instead of eight 4-row gathers.
              if (lane == 0) {
                const int key0 = meta.v[s];
                for (int cb = 0; cb < C::CB; ++cb) {
                  tma_load_4d(stage_k(st) + cb * C::KEYS * 128 + s * C::SUB * 128, &tm_k32, cb * C::EPB, h, key0, b,
                              kv_full(st));
                  tma_load_4d(stage_v(st) + cb * C::KEYS * 128 + s * C::SUB * 128, &tm_v32, cb * C::EPB, h, key0, b,
                              kv_full(st));
                }
              }
            } else if constexpr (GATHER) {
              // Lane i holds slot i's row; lanes 0-7 gather K rows 4j..4j+3, lanes 8-15 V rows.
              const int row = meta.v[s] * row_mul + row_base;
              const int j = lane & 7;
              const int r0 = __shfl_sync(0xffffffffu, row, 4 * j), r1 = __shfl_sync(0xffffffffu, row, 4 * j + 1);
              const int r2 = __shfl_sync(0xffffffffu, row, 4 * j + 2), r3 = __shfl_sync(0xffffffffu, row, 4 * j + 3);
              if (lane < 16) {
                const uint32_t dst = (lane < 8 ? stage_k(st) : stage_v(st)) + s * C::SUB * 128 + j * 512;
                const void* tm = lane < 8 ? static_cast<const void*>(&tm_k) : static_cast<const void*>(&tm_v);
                for (int cb = 0; cb < C::CB; ++cb)
                  tma_gather4(dst + cb * C::KEYS * 128, tm, cb * C::EPB, r0, r1, r2, r3, kv_full(st));
              }
            } else if (lane == 0) {
              const int key0 = meta.v[s] * C::SUB;
              for (int cb = 0; cb < C::CB; ++cb) {
                tma_load_4d(stage_k(st) + cb * C::KEYS * 128 + s * C::SUB * 128, &tm_k, cb * C::EPB, h, key0, b,
                            kv_full(st));
                tma_load_4d(stage_v(st) + cb * C::KEYS * 128 + s * C::SUB * 128, &tm_v, cb * C::EPB, h, key0, b,
                            kv_full(st));
              }
            }
            if (lane == 0) bulk_load(stage_bits(st) + s * 512, p.bits2 + static_cast<size_t>(t) * 128, 512, kv_full(st));
          }
        return true;
      };
      for (int c = 0; c < nch && ok; c += 2) {
        if (!(ok = issue_chunk(c, m0))) break;
        ++g;
        m0 = load_chunk_meta<C::CH, GATHER>(p.kb2, p.cols, t0, n_sub, c + 2, lane);
        if (c + 1 < nch) {
          if (!(ok = issue_chunk(c + 1, m1))) break;
          ++g;
          m1 = load_chunk_meta<C::CH, GATHER>(p.kb2, p.cols, t0, n_sub, c + 3, lane);
        }
      }
      if (!ok) break;
      ++qc;
    }
    if (!ok && lane == 0) {
      // Drain: wait (bounded, ignoring the abort flag) for every copy this warp issued.
      volatile int never = 0;
      for (uint32_t k = (g >= C::NS ? g - C::NS : 0); k < g; ++k)
        if (static_cast<long long>(k) != skipped) mbar_wait(kv_full(k % C::NS), (k / C::NS) & 1, &never, wlim);
      if (pending_q) mbar_wait(q_full, (qc & 1), &never, wlim);
    }
  } else if (warp == 1) {
    {
      // ------------------------------------------------------------------ MMA issuer
      // The whole warp runs the loop with warp-uniform descriptors and one elected lane issues each MMA / commit
      // (measured 6 % faster on the sparse configuration-3 backward than a lane-0 loop).
      auto wait_ = [&](uint32_t bar, uint32_t parity) -> bool { return warp_wait(bar, parity, abort_flag, wlim); };
      auto issue_ = [&](auto&& fn) {
        if (elect_one_sync()) fn();
        __syncwarp();
      };
      constexpr uint32_t kIdescPV = instr_desc(F32, 128, D, false, true);
      // 3xTF32: each product is hi*hi + hi*lo + lo*hi (the lo*lo term is below fp32 precision).
      constexpr int kPasses = X3 ? 3 : 1;
      const uint64_t qdesc = smem_desc(q_smem, 16, 1024), qlo_desc = smem_desc(q_lo, 16, 1024);
      uint32_t g = 0, qc = 0;
      bool ok = true;
      // The item's list range is read one item ahead (a dependent global load at each item start would stall).
      int nt0 = 0, nt1 = 0;
      if (blockIdx.x < p.n_items) {
        nt0 = __ldg(p.ptr2 + blockIdx.x % per_bh);
        nt1 = __ldg(p.ptr2 + blockIdx.x % per_bh + 1);
      }
      for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
        const int n_sub = nt1 - nt0;
        if (it + static_cast<int>(gridDim.x) < p.n_items) {
          nt0 = __ldg(p.ptr2 + (it + gridDim.x) % per_bh);
          nt1 = __ldg(p.ptr2 + (it + gridDim.x) % per_bh + 1);
        }
        const int nch = (n_sub + C::CH - 1) / C::CH;
        if (nch == 0) continue;
        if (!(ok = wait_((X3 && !C::Q_TMEM) ? q_ready : q_full, qc & 1))) break;
        if (lane == 0) FWN_TR(10, it);
        const uint32_t g0 = g;
        // S = Q K^T of chunk c (K / V must have landed and the S buffer must be free).
        auto issue_s = [&](int c) -> bool {
          const uint32_t gg = g0 + c;
          const int st = gg % C::NS, sb = gg & 1;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (lane == 0) FWN_TR(15, c);
          if (!wait_(X3 ? kv_ready(st) : kv_full(st), (gg / C::NS) & 1)) return false;
          if (lane == 0) FWN_TR(16, c);
          // The S buffer is free once the softmax has read it, or (P over S) once P V of chunk gg-2 is complete.
          if (!wait_(C::P_OVER_S ? p_empty(sb) : s_empty(sb), ((gg >> 1) & 1) ^ 1)) return false;
          if (lane == 0) FWN_TR(13, c);
          tc_fence_after();
          const uint32_t idesc_s = instr_desc(F32, 128, 32 * n_in, false, false);
          const uint64_t kdesc = smem_desc(stage_k(st), 16, 1024), klo_desc = smem_desc(stage_klo(st), 16, 1024);
  #pragma unroll
          for (int pass = 0; pass < kPasses; ++pass) {
  #pragma unroll
            for (int kk = 0; kk < D / C::KSTEP; ++kk) {
              const uint32_t cb = kk / 4, within = (kk % 4) * 32;
              const uint64_t a = (pass == 2 ? qlo_desc : qdesc) + ((cb * C::ROWS * 128 + within) >> 4);
              const uint64_t bd = (pass == 1 ? klo_desc : kdesc) + ((cb * C::KEYS * 128 + within) >> 4);
              if constexpr (C::Q_TMEM) {
                // A = Q in TMEM (3xTF32: its lo copy D columns on in the third pass): K = 8 tf32 elements = 8
                // columns per MMA.
                const uint32_t a_t = tmem + C::Q_COL + (pass == 2 ? D : 0) + 8 * kk;
                issue_([&] { mma_ts<true>(tmem + sb * C::S_STRIDE, a_t, bd, idesc_s, (pass > 0 || kk > 0) ? 1u : 0u); });
              } else {
                issue_([&] { mma_ss<F32>(tmem + sb * C::S_STRIDE, a, bd, idesc_s, (pass > 0 || kk > 0) ? 1u : 0u); });
              }
            }
          }
          issue_([&] {
            mma_commit(s_full(sb));
            if (c == nch - 1) mma_commit(q_empty);
          });
          if (lane == 0) FWN_TR(11, c);
          return true;
        };
        // O += P V of chunk c (P written by the softmax; O free once the previous item's epilogue read it).
        auto issue_pv = [&](int c) -> bool {
          const uint32_t gg = g0 + c;
          const int st = gg % C::NS, pbuf = gg & 1;
          const int n_in = min(C::CH, n_sub - C::CH * c);
          if (!wait_(p_full(pbuf), (gg >> 1) & 1)) return false;
          if (c == 0 && !wait_(o_empty, (qc & 1) ^ 1)) return false;
          if (lane == 0) FWN_TR(14, c);
          tc_fence_after();
          const int ksteps = n_in * C::SUB / C::KSTEP;
          // V: MN-major B (128-byte swizzle for bf16, the 32-byte-atom variant for tf32), hi and lo copies.
          const uint64_t vdesc = F32 ? smem_desc(stage_v(st), C::KEYS * 128, 512, kLayoutSW128Base32B)
                                     : smem_desc(stage_v(st), C::KEYS * 128, 1024);
          if constexpr (C::P_TMEM) {
            // P from TMEM: K = 16 bf16 keys (8 columns of packed pairs) or 8 tf32 keys (8 columns) per MMA.
            const uint32_t pcol = tmem + C::P_COL + C::P_STRIDE * pbuf;
            for (int kk = 0; kk < ksteps; ++kk) {
              const uint64_t bd = vdesc + ((kk * C::KSTEP * 128) >> 4);
              issue_([&] { mma_ts<F32>(tmem + C::O_COL, pcol + 8 * kk, bd, kIdescPV, (c == 0 && kk == 0) ? 0u : 1u); });
            }
          } else {
            // P in shared memory (K-major A), hi and lo copies.
            const uint64_t pdesc = smem_desc(p_smem(pbuf), 16, 1024), plo_desc = smem_desc(p_lo(pbuf), 16, 1024);
            const uint64_t vlo_desc = smem_desc(stage_vlo(st), C::KEYS * 128, 512, kLayoutSW128Base32B);
            for (int pass = 0; pass < kPasses; ++pass) {
              for (int kk = 0; kk < ksteps; ++kk) {
                const uint32_t cb = kk / 4, within = (kk % 4) * 32;
                const uint64_t a = (pass == 2 ? plo_desc : pdesc) + ((cb * C::ROWS * 128 + within) >> 4);
                const uint64_t bd = (pass == 1 ? vlo_desc : vdesc) + ((kk * C::KSTEP * 128) >> 4);
                issue_([&] {
                  mma_ss<F32>(tmem + C::O_COL, a, bd, kIdescPV, (c == 0 && pass == 0 && kk == 0) ? 0u : 1u);
                });
              }
            }
          }
          issue_([&] {
            mma_commit(p_empty(pbuf));
            mma_commit(kv_empty(st));
            if (c == nch - 1) mma_commit(o_full);
          });
          if (lane == 0) FWN_TR(12, c);
          return true;
        };
        // S of chunk c goes ahead of P V of chunk c-1, so that the tensor core overlaps the softmax.
        for (int c = 0; c <= nch && ok; ++c) {
          if (c < nch && !(ok = issue_s(c))) break;
          if (c >= 1 && !(ok = issue_pv(c - 1))) break;
        }
        g = g0 + nch;
        ++qc;
      }
      // Drain the tensor pipe before TMEM is released.
      issue_([&] { mma_commit(drain); });
      volatile int never = 0;
      mbar_wait(drain, 0, &never, wlim);
    }
  } else if (X3 && warp >= 6) {
    // ------------------------------------------------------------------ 3xTF32 converter (warps 6-9)
    const int ctid = threadIdx.x - 192;
    uint32_t g = 0, qc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh;
      const int n_sub = p.ptr2[pb + 1] - p.ptr2[pb];
      const int nch = (n_sub + C::CH - 1) / C::CH;
      if (nch == 0) continue;
      if constexpr (!C::Q_TMEM) {
        if (!(ok = mbar_wait(q_full, qc & 1, abort_flag, wlim))) break;
        split_tf32(q_smem, q_lo, C::Q_BYTES, ctid, 128);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_ready);
      }
      for (int c = 0; c < nch; ++c, ++g) {
        const int st = g % C::NS;
        if (!(ok = mbar_wait(kv_full(st), (g / C::NS) & 1, abort_flag, wlim))) break;
        split_tf32(stage_k(st), stage_klo(st), C::KV_BYTES, ctid, 128);
        split_tf32(stage_v(st), stage_vlo(st), C::KV_BYTES, ctid, 128);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(kv_ready(st));
      }
      ++qc;
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    uint32_t g = 0, qc = 0;
    bool ok = true;
    int nt0 = 0, nt1 = 0;  // list range, read one item ahead
    if (blockIdx.x < p.n_items) {
      nt0 = __ldg(p.ptr2 + blockIdx.x % per_bh);
      nt1 = __ldg(p.ptr2 + blockIdx.x % per_bh + 1);
    }
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh, bh = it / per_bh, h = bh % p.heads, b = bh / p.heads;
      const int n_sub = nt1 - nt0;
      if (it + static_cast<int>(gridDim.x) < p.n_items) {
        nt0 = __ldg(p.ptr2 + (it + gridDim.x) % per_bh);
        nt1 = __ldg(p.ptr2 + (it + gridDim.x) % per_bh + 1);
      }
      const int nch = (n_sub + C::CH - 1) / C::CH;
      const int qrow = pb * C::ROWS + row;
      float m_ref = -INFINITY, l = 0.f;
      if constexpr (C::Q_TMEM) {
        // The item's Q into TMEM (this thread's row into its lane), once the previous item's last S MMA is
        // complete; rows past n are zero (as the TMA load's out-of-range fill).
        if (nch > 0) {
          if (!(ok = mbar_wait(q_empty, (qc & 1) ^ 1, abort_flag, wlim))) break;
          tc_fence_after();
          const float* src = qrow < p.n ? static_cast<const float*>(p.q) + static_cast<int64_t>(b) * p.q_sb +
                                              static_cast<int64_t>(qrow) * p.q_sn + static_cast<int64_t>(h) * p.q_sh
                                        : nullptr;
#pragma unroll
          for (int j = 0; j < D / 32; ++j) {
            float v[32];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float4 x = src ? __ldg(reinterpret_cast<const float4*>(src + 32 * j) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
              v[4 * i] = x.x;
              v[4 * i + 1] = x.y;
              v[4 * i + 2] = x.z;
              v[4 * i + 3] = x.w;
            }
            if constexpr (X3) {
              // hi (13 low mantissa bits cleared) and lo = x - hi, D columns apart.
              float lo[32];
#pragma unroll
              for (int i = 0; i < 32; ++i) {
                const float hi = __uint_as_float(__float_as_uint(v[i]) & 0xFFFFE000u);
                lo[i] = v[i] - hi;
                v[i] = hi;
              }
              tmem_st32(trow + C::Q_COL + D + 32 * j, lo);
            }
            tmem_st32(trow + C::Q_COL + 32 * j, v);
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(q_full);
        }
      }
      const uint32_t g0 = g;
      for (int c = 0; c < nch; ++c) {
        const uint32_t gg = g0 + c;
        const int sb = gg & 1, st = gg % C::NS;
        const int n_in = min(C::CH, n_sub - C::CH * c);
        float s[C::KEYS];
        if (!(ok = mbar_wait(s_full(sb), (gg >> 1) & 1, abort_flag, wlim))) break;
        if (lane == 0) FWN_TR(20, c);
        tc_fence_after();
        tmem_ld32(trow + sb * C::S_STRIDE, *reinterpret_cast<float(*)[32]>(&s[0]));
        if constexpr (C::CH == 2) {
          if (n_in == 2) tmem_ld32(trow + sb * C::S_STRIDE + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
        }
        // While S is read from TMEM: the chunk's mask words (they land with its K / V tiles) and, for bf16, the
        // P buffer (free once P V of chunk gg-2 is complete).
        ok = mbar_wait(kv_full(st), (gg / C::NS) & 1, abort_flag, wlim);
        if (C::P_TMEM && !C::P_OVER_S && ok) ok = mbar_wait(p_empty(sb), ((gg >> 1) & 1) ^ 1, abort_flag, wlim);
        uint32_t w0 = 0u, w1 = 0u;
        if (ok) {
          w0 = ld_shared_u32(stage_bits(st) + row * 4);
          if constexpr (C::CH == 2) {
            if (n_in == 2) w1 = ld_shared_u32(stage_bits(st) + 512 + row * 4);
          }
        }
        tmem_wait_ld();
        reg_fence(s);
        if (!ok) break;
        if (lane == 0) FWN_TR(24, c);
        tc_fence_before();
        __syncwarp();
        if (!C::P_OVER_S && lane == 0) mbar_arrive(s_empty(sb));
        const uint32_t any0 = __reduce_or_sync(0xffffffffu, w0);
        const uint32_t any1 = C::CH == 2 ? __reduce_or_sync(0xffffffffu, w1) : 0u;
        // Columns are handled in groups of 8 (one 16-byte chunk of a bf16 P row); a group that no row
        // of the warp may attend to is skipped by the whole warp. Four independent partial maxima / sums
        // keep the dependency chains short.
        const float m_old = m_ref;
        bool grow = false;
        float corr = 1.f;
        // Exact two-pass update: masked row max, lazy rescale of the reference, then p = 2^(s - m).
        auto two_pass = [&](float (&e)[C::KEYS]) {
          float mxp[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
          for (int g = 0; g < C::KEYS / 8; ++g) {
            const uint32_t w = g < 4 ? w0 : w1;
            const uint32_t any = g < 4 ? any0 : any1;
            if ((any >> (8 * (g & 3))) & 0xFFu) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int j = 8 * g + i;
                mxp[i & 3] = (w & (1u << (j & 31))) ? fmaxf(mxp[i & 3], s[j]) : mxp[i & 3];
              }
            }
          }
          const float mx = fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3]));
          const float m_new = mx * p.scale_log2;
          if (l == 0.f) {
            m_ref = m_new;  // nothing accumulated yet (O row is 0): any reference will do
          } else if (m_new > m_ref + 8.0f) {
            grow = true;
            corr = ex2(m_old - m_new);
            m_ref = m_new;
            l *= corr;
          }
          const float neg_m = -m_ref;
          float lp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int g = 0; g < C::KEYS / 8; ++g) {
            const uint32_t w = g < 4 ? w0 : w1;
            const uint32_t any = g < 4 ? any0 : any1;
            if ((any >> (8 * (g & 3))) & 0xFFu) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int j = 8 * g + i;
                const float t = ex2(fmaf(s[j], p.scale_log2, neg_m));
                e[j] = (w & (1u << (j & 31))) ? t : 0.f;
                lp[i & 3] += e[j];
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) e[8 * g + i] = 0.f;
            }
          }
          l += (lp[0] + lp[1]) + (lp[2] + lp[3]);
        };
        if constexpr (!F32) {
          // One pass against the current reference, accepted while the row's chunk sum is at most 2^16 (so is
          // every p: bf16 P keeps its relative precision, the fp32 accumulators stay far from overflow). Rows
          // with nothing accumulated yet take this chunk's unmasked row max as their reference (an upper bound of
          // the allowed logits); they are accepted only if their sum is at least 2^-54 (their largest allowed p
          // is then at least 2^-60, so whatever underflowed is negligible). Otherwise the whole warp redoes the
          // chunk with the exact two-pass update. Paired f32x2 arithmetic for the scaling and the sums.
          uint32_t pk[C::KEYS / 2];
          float2 lp2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
          const bool fresh = l == 0.f;
          float m_use = m_ref;
          if (__any_sync(0xffffffffu, fresh)) {
            float up[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int j = 0; j < C::KEYS; ++j)
              if (j < 32 * n_in) up[j & 3] = fmaxf(up[j & 3], s[j]);
            const float umax = fmaxf(fmaxf(up[0], up[1]), fmaxf(up[2], up[3])) * p.scale_log2;
            if (fresh) m_use = umax;
          }
          const float2 sc2 = make_float2(p.scale_log2, p.scale_log2), nm2 = make_float2(-m_use, -m_use);
#pragma unroll
          for (int g = 0; g < C::KEYS / 8; ++g) {
            const uint32_t w = g < 4 ? w0 : w1;
            const uint32_t any = g < 4 ? any0 : any1;
            if ((any >> (8 * (g & 3))) & 0xFFu) {
#pragma unroll
              for (int i = 0; i < 8; i += 2) {
                const int j = 8 * g + i;
                const float2 x = ffma2(make_float2(s[j], s[j + 1]), sc2, nm2);
                const float t0 = ex2(x.x), t1 = ex2(x.y);
                const float e0 = (w & (1u << (j & 31))) ? t0 : 0.f;
                const float e1 = (w & (1u << ((j + 1) & 31))) ? t1 : 0.f;
                lp2[(i >> 1) & 1] = fadd2(lp2[(i >> 1) & 1], make_float2(e0, e1));
                pk[j >> 1] = pack_bf16(e0, e1);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 4; ++i) pk[4 * g + i] = 0u;
            }
          }
          const float sum = (lp2[0].x + lp2[0].y) + (lp2[1].x + lp2[1].y);
          const bool bad = !(sum <= 65536.f) ||
                           (fresh && (w0 | w1) != 0u && !(sum >= 5.5511151231257827e-17f));  // 2^-54
          if (__any_sync(0xffffffffu, bad)) {
            float e[C::KEYS];
            two_pass(e);
#pragma unroll
            for (int j = 0; j < C::KEYS / 2; ++j) pk[j] = pack_bf16(e[2 * j], e[2 * j + 1]);
          } else {
            m_ref = m_use;
            l += sum;
          }
          if (lane == 0) FWN_TR(26, c);
          // P -> TMEM (the buffer was released above); the row's packed pairs go to its lane.
          const uint32_t pcol = trow + C::P_COL + C::P_STRIDE * sb;
          tmem_st16(pcol, *reinterpret_cast<const uint32_t(*)[16]>(&pk[0]));
          if constexpr (C::CH == 2) {
            if (n_in == 2) tmem_st16(pcol + 16, *reinterpret_cast<const uint32_t(*)[16]>(&pk[16]));
          }
          tmem_wait_st();
        } else {
          float e[C::KEYS];
          two_pass(e);
          if (lane == 0) FWN_TR(26, c);
          if constexpr (C::P_TMEM) {
            // tf32 P -> TMEM (the buffer was released above), one 32-key tile at a time.
            const uint32_t pcol = trow + C::P_COL + C::P_STRIDE * sb;
            tmem_st32(pcol, *reinterpret_cast<const float(*)[32]>(&e[0]));
            if constexpr (C::CH == 2) {
              if (n_in == 2) tmem_st32(pcol + 32, *reinterpret_cast<const float(*)[32]>(&e[32]));
            }
            tmem_wait_st();
          }
          if constexpr (!C::P_TMEM) {
            // 3xTF32: P hi (13 low mantissa bits cleared) and lo = P - hi into shared memory.
            if (!(ok = mbar_wait(p_empty(sb), ((gg >> 1) & 1) ^ 1, abort_flag, wlim))) break;
            const uint32_t pbase = p_smem(sb);
#pragma unroll
            for (int cc = 0; cc < 16; ++cc) {
              if (cc < 8 * n_in) {
                const int blk = cc >> 3, ch = cc & 7;
                const uint32_t off = blk * C::ROWS * 128 + sw128_offset(row, ch);
                uint32_t h[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                  h[i] = __float_as_uint(e[4 * cc + i]) & 0xFFFFE000u;
                  lo[i] = __float_as_uint(e[4 * cc + i] - __uint_as_float(h[i]));
                }
                st_shared_v4(pbase + off, h[0], h[1], h[2], h[3]);
                st_shared_v4(p_lo(sb) + off, lo[0], lo[1], lo[2], lo[3]);
              }
            }
          }
        }
        if constexpr (!C::P_TMEM) fence_proxy_async_smem();  // shared-memory P -> tensor core reads
        if (lane == 0) FWN_TR(27, c);
        // Rescale O rows whose reference max grew (only rows that accumulated something: grow needs l > 0).
        const bool rescale = grow;
        if (__any_sync(0xffffffffu, rescale)) {
          const uint32_t prev = gg - 1;
          if (lane == 0) FWN_TR(28, c);
          if (!(ok = mbar_wait(p_empty(prev & 1), (prev >> 1) & 1, abort_flag, wlim))) break;
          tc_fence_after();
#pragma unroll
          for (int j = 0; j < D / 32; ++j) {
            float o[32];
            tmem_ld32(trow + C::O_COL + 32 * j, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= corr;
            tmem_st32(trow + C::O_COL + 32 * j, o);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(sb));
        if (lane == 0) FWN_TR(21, c);
      }
      if (!ok) break;
      g = g0 + nch;
      // ---------------------------------------------------------------- epilogue
      const bool has = l > 0.f;
      const float inv = has ? 1.f / l : 0.f;
      if (p.lse != nullptr) {
        const float lse = has ? (m_ref + lg2(l)) * 0.69314718055994530942f : -INFINITY;
        p.lse[static_cast<size_t>(bh) * p.lse_rows + qrow] = lse;
      }
      const bool store = qrow < p.n;
      uint8_t* orow = reinterpret_cast<uint8_t*>(p.o) +
                      (static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(qrow) * p.o_sn +
                       static_cast<int64_t>(h) * p.o_sh) * C::ES;
      if (nch == 0) {
        if (store) {
          for (int i = 0; i < D * C::ES / 16; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      if (!(ok = mbar_wait(o_full, qc & 1, abort_flag, wlim))) break;
      if (lane == 0) FWN_TR(22, it);
      tc_fence_after();
#pragma unroll
      for (int j = 0; j < D / 32; ++j) {
        float o[32];
        tmem_ld32(trow + C::O_COL + 32 * j, o);
        tmem_wait_ld();
        if (store) {
          if constexpr (!F32) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              reinterpret_cast<uint4*>(orow + j * 64)[i] =
                  make_uint4(pack_bf16(o[8 * i] * inv, o[8 * i + 1] * inv), pack_bf16(o[8 * i + 2] * inv, o[8 * i + 3] * inv),
                             pack_bf16(o[8 * i + 4] * inv, o[8 * i + 5] * inv), pack_bf16(o[8 * i + 6] * inv, o[8 * i + 7] * inv));
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              reinterpret_cast<float4*>(orow + j * 128)[i] =
                  make_float4(o[4 * i] * inv, o[4 * i + 1] * inv, o[4 * i + 2] * inv, o[4 * i + 3] * inv);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_empty);
      if (lane == 0) FWN_TR(23, it);
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
