// Backward kernels of the block-sparse masked flash attention (sm_100a, tcgen05 + TMA).
//
// Replaces _attention_bwd with _bwd_dq_kernel / _bwd_dkv_kernel (src/faster_weathernext/pallas_attn.py:
// 161-215, 274-311). Same algorithm: delta = rowsum(O * dO) first; then P is recomputed tile by tile
// from the forward's log-sum-exp, P = where(valid, exp(S - lse), 0), dS = P * (dP - delta), and
//   dQ  = scale * sum dS K        per query block over the forward list
//   dK  = scale * sum dS^T Q,  dV = sum P^T dO
//                                 per key block over the transposed list
// so every output row is owned by one CTA: no atomics, deterministic (as pallas_attn.py:297-311).
//
// One kernel template serves every pass ("kind"): "rows" are the 128 rows of the work item (queries for
// dQ, keys otherwise) held in shared memory for the whole item (R0, R1), "columns" are walked in chunks of
// CH 32-wide tiles (C0, C1):
//               dQ          dK/dV        dV only      dK only
//   R0, R1      Q, dO       K, V         K            K, V
//   C0, C1      K, V        Q, dO        Q, dO        Q, dO
//   S  = R0 C0^T            always
//   dP = R1 C1^T            dQ, dK/dV, dK only
//   acc0 += dS C0           dQ, dK/dV, dK only   (MN-major B)
//   acc1 += P  C1           dK/dV, dV only       (MN-major B)
// dV only + dK only replace the dK/dV pass where it does not fit one CTA: 3xTF32 (hi / lo operand copies) and
// tf32 at head_dim 128 (shared memory), bf16 at head_dim 128 (the TMEM columns of a CTA that shares its SM).
// Roles: warp 0 TMA producer; warp 1 TMEM allocation + single-thread MMA issue;
// warps 2-5 the elementwise stage (thread = row = TMEM lane) and the epilogue; in 3xTF32 warps 6-9 split
// every landed tile into hi (in place) and lo copies. S / dP of chunk c+1 are issued before the
// accumulating MMAs of chunk c. tf32 operands read MN-major use a second copy of the column tile with
// the 32-byte-atom swizzle (SWIZZLE_128B_BASE32B).
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace fwn {

enum BwdKind : int { kBwdDQ = 0, kBwdDKV = 1, kBwdDV = 2, kBwdDK = 3 };

struct BwdParams {
  const int32_t* ptr2;
  const int32_t* kb2;     // tile mode: column block of each tile
  const int32_t* cols;    // gathered mode: column of each slot [T * 32]
  const uint32_t* bits2;
  int head_major;         // gathered mode: rows of the 2D column-operand views are (b, h, node)
  const float* lse;    // [B, H, lse_rows] natural log
  const float* delta;  // [B, H, lse_rows]
  void* out0;          // dQ or dK (kinds with acc0)
  void* out1;          // dV (kinds with acc1)
  int64_t o_sb, o_sn, o_sh;
  int heads, n, np, lse_rows, n_items;
  float scale;         // softmax scale (applied to acc0)
  float scale_log2;    // scale * log2(e)
  unsigned long long* trace;  // FWN_TRACE builds: event records (else unused)
  // Row operands and their element strides (read by the elementwise warps where the rows live in TMEM).
  const void* r0;
  const void* r1;
  int64_t r0_sb, r0_sn, r0_sh, r1_sb, r1_sn, r1_sh;
};

template <int KIND, int D, bool F32, int CH, bool X3>
struct BwdCfg {
  static constexpr bool ROWS_ARE_KEYS = KIND != kBwdDQ;
  static constexpr bool NEED_DP = KIND != kBwdDV;
  static constexpr bool ACC_DS = KIND != kBwdDV;
  static constexpr bool ACC_P = KIND == kBwdDKV || KIND == kBwdDV;
  static constexpr int ES = F32 ? 4 : 2;
  static constexpr int EPB = 128 / ES;
  static constexpr int CB = D / EPB;
  static constexpr int ROWS = 128;
  static constexpr int SUB = 32;
  static constexpr int COLS = 32 * CH;       // columns per chunk
  static constexpr int KSTEP = F32 ? 8 : 16;
  static constexpr int XL = X3 ? 2 : 1;      // copies of an operand: hi (in place) and lo
  // Row operands: R0, R1 (dP needs R1).
  static constexpr int NR = NEED_DP ? 2 : 1;
  // Column tiles per stage: C0 (K-major), C1 (K-major for dP; bf16 also serves as dV's MN-major B),
  // C0 MN-major copy (tf32, for acc0), C1 MN-major copy (tf32, for acc1); then lo copies (3xTF32).
  static constexpr bool LOAD_C1 = NEED_DP || (ACC_P && !F32);
  static constexpr bool LOAD_C0MN = F32 && ACC_DS;
  static constexpr bool LOAD_C1MN = F32 && ACC_P;
  static constexpr int SLOT_C1 = 1;
  static constexpr int SLOT_C0MN = 1 + (LOAD_C1 ? 1 : 0);
  static constexpr int SLOT_C1MN = SLOT_C0MN + (LOAD_C0MN ? 1 : 0);
  static constexpr int NC = SLOT_C1MN + (LOAD_C1MN ? 1 : 0);
  // dS / P (bf16 packed pairs, or fp32) go to TMEM over the S / dP columns they are computed from, and the
  // accumulating MMAs read them as the A operand from tensor memory; S / dP are double-buffered (one 32-wide tile
  // per chunk), so the elementwise stage of chunk c overlaps the S / dP MMAs of chunk c+1. 3xTF32 passes have one
  // of dS / P: its hi copy goes over S, its lo copy over dP. (The shared-memory dS / P path below serves no
  // configuration now and is kept for kernels whose TMEM would not hold two buffers.)
  static constexpr bool G_TMEM = true;
  // One stage where the hi / lo (3xTF32) or fp32 head_dim-128 operands leave room for no second one.
  static constexpr bool BIG = X3 || (F32 && D == 128);
  // dS / P rows of 32 bf16 columns are 64 bytes: 64-byte swizzle (half the shared memory of a 128-byte row).
  static constexpr bool G64 = COLS * ES == 64;
  static constexpr int R_BYTES = CB * ROWS * 128;       // one row operand
  // tf32 (one CTA per SM): the row operands live in TMEM, one fp32 element per column (the A operands of S / dP,
  // loaded by the elementwise warps: thread = row = lane); shared memory then holds only column stages (at head_dim
  // 128 four instead of two for the dQ / dK passes), and the S / dP MMAs read a fifth of the shared-memory bytes.
  // 3xTF32: the first row operand in TMEM (hi and lo copies, split by the elementwise warps); the second stays in
  // shared memory, split there by the converter warps.
  static constexpr int NR_TMEM = X3 ? 1 : F32 ? NR : 0;
  static constexpr int NR_SMEM = NR - NR_TMEM;
  static constexpr bool R_TMEM = NR_TMEM > 0;
  static constexpr int R_COLS = NR_TMEM * D * XL;
  static constexpr int C_BYTES = CB * COLS * 128;       // one column operand per stage
  static constexpr int BITS_OFF = NC * XL * C_BYTES;
  // lse / delta of the columns (rows are keys): lse times log2 e where the producer stores them through registers
  // (gathered mode), the natural-log values where they are bulk-copied (tile mode).
  static constexpr int VEC_OFF = BITS_OFF + CH * 512;
  static constexpr int STAGE_RAW = VEC_OFF + (ROWS_ARE_KEYS ? CH * 256 : 0);
  static constexpr int STAGE_BYTES = (STAGE_RAW + 1023) / 1024 * 1024;
  static constexpr int G_BYTES = G_TMEM ? 0 : G64 ? ROWS * 64 : (COLS * ES / 128) * ROWS * 128;  // one dS (or P) tile
  static constexpr int NG = (ACC_DS ? 1 : 0) + (ACC_P ? 1 : 0);        // dS, P tiles per buffer
  static constexpr int ACC_COLS = (ACC_DS ? D : 0) + (ACC_P ? D : 0);  // TMEM columns of the accumulators
  // TMEM S / dP buffers: S (32 CH columns) then dP; as many as the accumulators leave room for in 256 columns
  // (bf16, two CTAs per SM) or 512 (tf32, one), at most 3 (bf16) or 4; 3xTF32 one.
  static constexpr int SD_W = 32 * CH;
  static constexpr int SD_STRIDE = 2 * SD_W;
  // bf16 dQ at head_dim 64 (the sparse configurations) runs four CTAs per SM with 128 TMEM columns each (QUAD): the
  // dQ accumulator and one S / dP buffer.
  static constexpr bool QUAD = !F32 && D == 64 && KIND == kBwdDQ;
  static constexpr int TMEM_MAX = F32 ? 512 : QUAD ? 128 : 256;
  static constexpr int NSD_FIT = (TMEM_MAX - R_COLS - ACC_COLS) / SD_STRIDE;
  static constexpr int NSD = !G_TMEM ? 1 : NSD_FIT < (F32 ? 4 : 3) ? NSD_FIT : (F32 ? 4 : 3);
  // dS / P buffers: the TMEM S / dP buffers (bf16); in shared memory one where two would not fit (3xTF32 except
  // dV only), else two.
  static constexpr int NB = G_TMEM ? NSD : (X3 && KIND != kBwdDV) ? 1 : 2;
  static constexpr int SDB = NSD < 2 ? 2 : NSD;  // barrier slots: sd_full / sd_empty, or one sd_full per buffer
  static constexpr int n_bar(int ns) { return 2 + 2 * ns + SDB + 2 * NB + 2 + 1 + (X3 ? 1 + ns : 0); }
  // + 1 KB of slack to align the dynamic shared memory base up to 1024 bytes; 3xTF32, whose second stage would
  // miss by a few hundred bytes, sizes it to the byte and checks the alignment at run time instead.
  static constexpr int SLACK = X3 ? 0 : 1024;
  static constexpr int smem_bytes(int ns) {
    return NR_SMEM * XL * R_BYTES + ns * STAGE_BYTES + NB * NG * XL * G_BYTES + n_bar(ns) * 8 + 16 + SLACK;
  }
  // bf16 shares an SM between two CTAs; tf32 and 3xTF32 have one.
  static constexpr int fit(int ns) {
    return smem_bytes(ns) <= (F32 ? 227 * 1024 : QUAD ? 227 * 1024 / 4 : 227 * 1024 / 2);
  }
  // Column stages: as many as fit (at most 8), so that the copies of the next chunks are in flight during the
  // elementwise stage; 3xTF32 one or two.
  static constexpr int NS = fit(8) ? 8 : fit(6) ? 6 : fit(4) ? 4 : fit(3) ? 3 : fit(2) ? 2 : 1;
  static constexpr int OFF_C = NR_SMEM * XL * R_BYTES;
  static constexpr int OFF_G = OFF_C + NS * STAGE_BYTES;
  static constexpr int OFF_BAR = OFF_G + NB * NG * XL * G_BYTES;
  // r_full/empty, c_full/empty, sd_full/empty, g_full/empty, acc_full/empty, drain; 3xTF32: r_ready, c_ready.
  static constexpr int N_BAR = n_bar(NS);
  static constexpr int SMEM_BYTES = OFF_BAR + N_BAR * 8 + 16 + SLACK;
  // TMEM: S / dP buffer b at column SD_STRIDE b (S) and SD_STRIDE b + SD_W (dP) with P / dS over them (tile j of
  // the chunk at + GW j: bf16 packed pairs, tf32 fp32); 3xTF32 S at 0 and dP at 64; then the accumulators.
  static constexpr int DP_OFF = G_TMEM ? SD_W : 64;
  static constexpr int GW = F32 ? 32 : 16;  // TMEM columns of one 32-wide tile's dS or P (fp32, or bf16 pairs)
  static constexpr int SD0 = R_COLS;  // first S / dP buffer column (after row operands in TMEM)
  static constexpr int ACC0 = G_TMEM ? SD0 + SD_STRIDE * NSD : 128;
  static constexpr int ACC1 = ACC0 + (ACC_DS ? D : 0);
  static constexpr int TMEM_NEED = ACC0 + ACC_COLS;
  static constexpr int TMEM_COLS = QUAD ? 128 : TMEM_NEED <= 256 ? 256 : 512;
  static constexpr int THREADS = X3 ? 320 : 192;
  static constexpr int MIN_BLOCKS = QUAD ? 4 : (2 * SMEM_BYTES <= 227 * 1024 && TMEM_COLS <= 256 && !X3) ? 2 : 1;
  static_assert(!(F32 && D == 128) || KIND != kBwdDKV, "tf32 head_dim 128: dV and dK run as separate passes");
  // Each SM sub-partition has 16,384 registers and takes a quarter of the resident warps (rounded up):
  // twelve warps (two CTAs) or ten (3xTF32) leave 168 per thread.
  // Four CTAs (24 warps, six per sub-partition) leave 85: 80 in units of 8.
  static constexpr int MAX_REGS = QUAD ? 80 : (MIN_BLOCKS == 2 || X3) ? 168 : 255;
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(G64 || COLS * ES % 128 == 0, "dS rows must fill 64-byte or whole 128-byte column blocks");
  static_assert(!G64 || (!F32 && CH == 1), "64-byte dS rows hold 32 bf16 columns");
  static_assert(!X3 || F32, "3xTF32 takes float32 operands");
  static_assert(NC <= 4, "at most four column operands per stage (one producer lane octet each)");
  static_assert(!G_TMEM || ((NSD >= 2 || QUAD) && TMEM_NEED <= TMEM_MAX),
                "TMEM dS / P: two S / dP buffers (QUAD: one) and the accumulators");
  static_assert(!QUAD || (NSD == 1 && TMEM_NEED <= 128 && MIN_BLOCKS * SMEM_BYTES <= 227 * 1024), "QUAD layout");
  static_assert(!(G_TMEM && X3) || (CH == 1 && NG == 1), "3xTF32 TMEM dS / P: one of dS / P, 32-wide tiles");
  static_assert(F32 || TMEM_NEED <= 256, "bf16: two CTAs per SM");
  static_assert(!R_TMEM || (G_TMEM && MIN_BLOCKS == 1), "TMEM row operands: one CTA per SM");
  static_assert(SMEM_BYTES == smem_bytes(NS), "shared memory layout");
};

// delta[b, h, r] = sum_d O[b, r, h, d] * dO[b, r, h, d] (fp32); rows r in [n, lse_rows) get 0.
// HBM-bound: each lane loads 16 bytes of O and of dO, a row is LPR consecutive lanes (a 128- or
// 256-byte row), so one warp reads 32 x 16 bytes of each tensor per step, fully coalesced.
template <bool F32, int D>
__global__ void __launch_bounds__(256) delta_kernel(const void* __restrict__ o, const void* __restrict__ d_o,
                                                    float* __restrict__ delta, int heads, int n, int lse_rows,
                                                    int64_t sb, int64_t sn, int64_t sh, int total_rows) {
  constexpr int ES = F32 ? 4 : 2;
  constexpr int LPR = D * ES / 16;          // lanes per row
  constexpr int RPW = 32 / LPR;             // rows per warp
  grid_dependency_wait();  // o comes from the forward (launched with programmatic serialization)
  allow_dependents();
  const int gwarp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int row_id = gwarp * RPW + lane / LPR, part = lane % LPR;
  float acc = 0.f;
  if (row_id < total_rows) {
    const int r = row_id % lse_rows, bh = row_id / lse_rows, h = bh % heads, b = bh / heads;
    if (r < n) {
      const int64_t off = (static_cast<int64_t>(b) * sb + static_cast<int64_t>(r) * sn + static_cast<int64_t>(h) * sh) * ES +
                          part * 16;
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(o) + off));
      const uint4 c = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(d_o) + off));
      if constexpr (F32) {
        acc = __uint_as_float(a.x) * __uint_as_float(c.x) + __uint_as_float(a.y) * __uint_as_float(c.y) +
              __uint_as_float(a.z) * __uint_as_float(c.z) + __uint_as_float(a.w) * __uint_as_float(c.w);
      } else {
        const uint32_t av[4] = {a.x, a.y, a.z, a.w}, cv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&av[i]));
          const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&cv[i]));
          acc += x.x * y.x + x.y * y.y;
        }
      }
    }
  }
#pragma unroll
  for (int d = LPR / 2; d > 0; d >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, d);
  if (part == 0 && row_id < total_rows) delta[row_id] = acc;
}

template <int KIND, int D, bool F32, int CH, bool GATHER, bool X3>
__global__ void __launch_bounds__(BwdCfg<KIND, D, F32, CH, X3>::THREADS) __maxnreg__((BwdCfg<KIND, D, F32, CH, X3>::MAX_REGS))
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_r0, const __grid_constant__ CUtensorMap tm_r1,
                    const __grid_constant__ CUtensorMap tm_c0, const __grid_constant__ CUtensorMap tm_c1,
                    const __grid_constant__ CUtensorMap tm_c0mn, const __grid_constant__ CUtensorMap tm_c1mn,
                    const __grid_constant__ CUtensorMap tm_c0r, const __grid_constant__ CUtensorMap tm_c1r,
                    const __grid_constant__ CUtensorMap tm_c0mnr, const __grid_constant__ CUtensorMap tm_c1mnr,
                    const BwdParams p) {
  // tm_c*r: 4D maps of 32-row boxes (gathered mode: tiles whose 32 columns are consecutive).
  using C = BwdCfg<KIND, D, F32, CH, X3>;
  extern __shared__ uint8_t smem_bwd[];
  uint8_t* smem = C::SLACK ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_bwd) + 1023) & ~uintptr_t(1023))
                           : smem_bwd;
  const uint32_t sbase = smem_u32(smem);
  if (sbase & 1023u) {
    // No slack and an unaligned base: the tile layouts need 1024-byte alignment; report and leave (uniformly,
    // before any wait).
    if (threadIdx.x == 0) atomicOr(&g_device_error, 0x100u);
    return;
  }
  // Row operand i (hi, or the operand itself), its lo copy at +NR; column slot s of a stage, lo copy at +NC.
  // Row operand i >= NR_TMEM (the ones in shared memory), its lo copy at +NR_SMEM.
  auto r_op = [&](int i, int lo) { return sbase + (lo * C::NR_SMEM + (i - C::NR_TMEM)) * C::R_BYTES; };
  auto stage = [&](int s) { return sbase + C::OFF_C + s * C::STAGE_BYTES; };
  auto slot = [&](uint32_t sb, int s, int lo) { return sb + (lo * C::NC + s) * C::C_BYTES; };
  auto g_tile = [&](int b, int which, int lo) {
    return sbase + C::OFF_G + ((b * C::NG + which) * C::XL + lo) * C::G_BYTES;
  };
  constexpr int G_DS = 0, G_P = C::ACC_DS ? 1 : 0;  // dS / P tile index within a buffer
  const uint32_t bar0 = sbase + C::OFF_BAR;
  const uint32_t r_full = bar0, r_empty = bar0 + 8;
  auto c_full = [&](int s) { return bar0 + 16 + 8 * s; };
  auto c_empty = [&](int s) { return bar0 + 16 + 8 * (C::NS + s); };
  const uint32_t bar1 = bar0 + 16 + 16 * C::NS;
  // One S / dP buffer (sd_full, sd_empty) or, with dS / P in TMEM, NSD (sd_full_b(b); a buffer is free again once
  // the accumulating MMAs that read its dS / P are complete: g_empty).
  const uint32_t sd_full = bar1, sd_empty = bar1 + 8;
  auto sd_full_b = [&](int b) { return bar1 + 8 * b; };
  auto g_full = [&](int b) { return bar1 + 8 * C::SDB + 8 * b; };
  auto g_empty = [&](int b) { return bar1 + 8 * C::SDB + 8 * (C::NB + b); };
  const uint32_t bar2 = bar1 + 8 * C::SDB + 16 * C::NB;
  const uint32_t acc_full = bar2, acc_empty = bar2 + 8, drain = bar2 + 16;
  // 3xTF32: the converter's "split done" barriers; the MMA waits on these instead of the TMA ones.
  const uint32_t r_ready = bar2 + 24;
  auto c_ready = [&](int s) { return bar2 + 32 + 8 * s; };
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + C::N_BAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + C::N_BAR * 8 + 4);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int trace_count = 0;  // FWN_TRACE builds: this lane's event count
#define FWN_TR(code, arg) trace_event(p.trace, trace_count, (code), (arg))
  if (threadIdx.x == 0) {
    mbar_init(r_full, (C::NR_TMEM > 0 ? 4 : 0) + (C::NR_SMEM > 0 ? 1 : 0));
    mbar_init(r_empty, 1);
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(c_full(s), (GATHER && C::ROWS_ARE_KEYS) ? 2 : 1);
      mbar_init(c_empty(s), 1);
    }
    if constexpr (C::G_TMEM) {
      for (int b = 0; b < C::NSD; ++b) mbar_init(sd_full_b(b), 1);
    } else {
      mbar_init(sd_full, 1);
      mbar_init(sd_empty, 4);
    }
    for (int b = 0; b < C::NB; ++b) {
      mbar_init(g_full(b), 4);
      mbar_init(g_empty(b), 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 4);
    mbar_init(drain, 1);
    if constexpr (X3) {
      mbar_init(r_ready, 4);
      for (int s = 0; s < C::NS; ++s) mbar_init(c_ready(s), 4);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_r0);
    if (C::NR == 2) tma_prefetch_desc(&tm_r1);
    tma_prefetch_desc(&tm_c0);
    if (C::LOAD_C1) tma_prefetch_desc(&tm_c1);
    if (C::LOAD_C0MN) tma_prefetch_desc(&tm_c0mn);
    if (C::LOAD_C1MN) tma_prefetch_desc(&tm_c1mn);
    if (GATHER) {
      tma_prefetch_desc(&tm_c0r);
      if (C::LOAD_C1) tma_prefetch_desc(&tm_c1r);
      if (C::LOAD_C0MN) tma_prefetch_desc(&tm_c0mnr);
      if (C::LOAD_C1MN) tma_prefetch_desc(&tm_c1mnr);
    }
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;
  const int per_bh = p.np;
  // Launched with programmatic serialization after the delta pass: its prologue above (barriers, TMEM, descriptor
  // prefetch) may overlap the delta pass; nothing the earlier kernels wrote is read before this.
  grid_dependency_wait();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (whole warp)
    // Tile metadata is prefetched two chunks ahead, and the next item's list range one item ahead.
    uint32_t g = 0, qc = 0;
    bool ok = true;
    int pending_r = 0;
    constexpr uint32_t kColBytes = C::SUB * D * C::ES;  // one 32-wide tile of one column operand
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
      const int nch = (n_sub + CH - 1) / CH;
      if (nch == 0) continue;
      ChunkMeta<CH> m0 = load_chunk_meta<CH, GATHER>(p.kb2, p.cols, t0, n_sub, 0, lane);
      ChunkMeta<CH> m1 = load_chunk_meta<CH, GATHER>(p.kb2, p.cols, t0, n_sub, 1, lane);
      if constexpr (C::NR_SMEM > 0) {
        // The row operands that live in shared memory.
        if (!(ok = mbar_wait(r_empty, (qc & 1) ^ 1, abort_flag))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(r_full, C::NR_SMEM * C::R_BYTES);
          for (int cb = 0; cb < C::CB; ++cb) {
            for (int op = C::NR_TMEM; op < C::NR; ++op)
              tma_load_4d(r_op(op, 0) + cb * C::ROWS * 128, op == 0 ? &tm_r0 : &tm_r1, cb * C::EPB, h, pb * C::ROWS, b,
                          r_full);
          }
        }
        pending_r = 1;
      }
      const int row_base = p.head_major ? (b * p.heads + h) * p.n : b * p.n * p.heads + h;
      const int row_mul = p.head_major ? 1 : p.heads;
      // Chunk c's copies; `meta` was loaded two chunks earlier. The loop below is unrolled by two so that
      // each prefetched register pair is consumed in place (a register move would wait for the load).
      auto issue_chunk = [&](int c, const ChunkMeta<CH>& meta) -> bool {
          const int st = g % C::NS;
          const int n_in = min(CH, n_sub - CH * c);
          // Gathered key rows: the lse / delta of the chunk's gathered queries go to shared memory through the
          // lanes' registers; their loads are issued before the stage wait so that their latency overlaps it.
          float vec_lse[CH], vec_delta[CH];
          if constexpr (GATHER && C::ROWS_ARE_KEYS) {
  #pragma unroll
            for (int s = 0; s < CH; ++s) {
              if (s < n_in) {
                const size_t vo = static_cast<size_t>(bh) * p.lse_rows + meta.v[s];
                vec_lse[s] = __ldg(p.lse + vo) * 1.4426950408889634f;  // log2 units for the elementwise warps
                vec_delta[s] = __ldg(p.delta + vo);
              }
            }
          }
          if (!mbar_wait(c_empty(st), ((g / C::NS) & 1) ^ 1, abort_flag)) return false;
          if (lane == 0) FWN_TR(3, c);
          // Gathered key rows: lse / delta of the gathered queries are stored by the lanes, not copied.
          const uint32_t per_tile = C::NC * kColBytes + 512 + ((C::ROWS_ARE_KEYS && !GATHER) ? 256 : 0);
          if (lane == 0) mbar_arrive_expect_tx(c_full(st), n_in * per_tile);
          __syncwarp();
          const uint32_t sb = stage(st);
  #pragma unroll
          for (int s = 0; s < CH; ++s) {
            if (s >= n_in) break;
            const int t = t0 + CH * c + s;
            if constexpr (GATHER) {
              const int col = meta.v[s];
              const int row = col * row_mul + row_base;
              const int j = lane & 7, which = lane >> 3;  // which: the column slot this lane octet loads
              const int r0 = __shfl_sync(0xffffffffu, row, 4 * j), r1 = __shfl_sync(0xffffffffu, row, 4 * j + 1);
              const int r2 = __shfl_sync(0xffffffffu, row, 4 * j + 2), r3 = __shfl_sync(0xffffffffu, row, 4 * j + 3);
              const int col0 = __shfl_sync(0xffffffffu, col, 0);
              if (__all_sync(0xffffffffu, col == col0 + lane)) {
                // The tile's 32 columns are consecutive: one 32-row box per slot and column block.
                if (lane == 0) {
                  for (int cb = 0; cb < C::CB; ++cb) {
                    const uint32_t off = cb * C::COLS * 128 + s * C::SUB * 128;
                    tma_load_4d(slot(sb, 0, 0) + off, &tm_c0r, cb * C::EPB, h, col0, b, c_full(st));
                    if (C::LOAD_C1)
                      tma_load_4d(slot(sb, C::SLOT_C1, 0) + off, &tm_c1r, cb * C::EPB, h, col0, b, c_full(st));
                    if (C::LOAD_C0MN)
                      tma_load_4d(slot(sb, C::SLOT_C0MN, 0) + off, &tm_c0mnr, cb * C::EPB, h, col0, b, c_full(st));
                    if (C::LOAD_C1MN)
                      tma_load_4d(slot(sb, C::SLOT_C1MN, 0) + off, &tm_c1mnr, cb * C::EPB, h, col0, b, c_full(st));
                  }
                }
              } else if (which < C::NC) {
                const void* tm = which == 0                                  ? static_cast<const void*>(&tm_c0)
                                 : (C::LOAD_C1 && which == C::SLOT_C1)       ? static_cast<const void*>(&tm_c1)
                                 : (C::LOAD_C0MN && which == C::SLOT_C0MN)   ? static_cast<const void*>(&tm_c0mn)
                                                                             : static_cast<const void*>(&tm_c1mn);
                const uint32_t dst = slot(sb, which, 0) + s * C::SUB * 128 + j * 512;
                for (int cb = 0; cb < C::CB; ++cb)
                  tma_gather4(dst + cb * C::COLS * 128, tm, cb * C::EPB, r0, r1, r2, r3, c_full(st));
              }
            } else if (lane == 0) {
              const int col0 = meta.v[s] * C::SUB;
              for (int cb = 0; cb < C::CB; ++cb) {
                const uint32_t off = cb * C::COLS * 128 + s * C::SUB * 128;
                tma_load_4d(slot(sb, 0, 0) + off, &tm_c0, cb * C::EPB, h, col0, b, c_full(st));
                if (C::LOAD_C1) tma_load_4d(slot(sb, C::SLOT_C1, 0) + off, &tm_c1, cb * C::EPB, h, col0, b, c_full(st));
                if (C::LOAD_C0MN)
                  tma_load_4d(slot(sb, C::SLOT_C0MN, 0) + off, &tm_c0mn, cb * C::EPB, h, col0, b, c_full(st));
                if (C::LOAD_C1MN)
                  tma_load_4d(slot(sb, C::SLOT_C1MN, 0) + off, &tm_c1mn, cb * C::EPB, h, col0, b, c_full(st));
              }
              if (C::ROWS_ARE_KEYS) {
                const size_t vo = static_cast<size_t>(bh) * p.lse_rows + col0;
                bulk_load(sb + C::VEC_OFF + s * 256, p.lse + vo, 128, c_full(st));
                bulk_load(sb + C::VEC_OFF + s * 256 + 128, p.delta + vo, 128, c_full(st));
              }
            }
            if (lane == 0) bulk_load(sb + C::BITS_OFF + s * 512, p.bits2 + static_cast<size_t>(t) * 128, 512, c_full(st));
          }
          if constexpr (GATHER && C::ROWS_ARE_KEYS) {
            // Second arrival of c_full: publishes the lanes' lse / delta stores.
  #pragma unroll
            for (int s = 0; s < CH; ++s) {
              if (s < n_in) {
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(sb + C::VEC_OFF + s * 256 + lane * 4), "f"(vec_lse[s])
                             : "memory");
                asm volatile("st.shared.f32 [%0], %1;" ::"r"(sb + C::VEC_OFF + s * 256 + 128 + lane * 4),
                             "f"(vec_delta[s])
                             : "memory");
              }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(c_full(st));
          }
        return true;
      };
      for (int c = 0; c < nch && ok; c += 2) {
        if (!(ok = issue_chunk(c, m0))) break;
        ++g;
        m0 = load_chunk_meta<CH, GATHER>(p.kb2, p.cols, t0, n_sub, c + 2, lane);
        if (c + 1 < nch) {
          if (!(ok = issue_chunk(c + 1, m1))) break;
          ++g;
          m1 = load_chunk_meta<CH, GATHER>(p.kb2, p.cols, t0, n_sub, c + 3, lane);
        }
      }
      if (!ok) break;
      ++qc;
    }
    if (!ok && lane == 0) {
      volatile int never = 0;
      for (uint32_t k = (g >= C::NS ? g - C::NS : 0); k < g; ++k)
        mbar_wait(c_full(k % C::NS), (k / C::NS) & 1, &never);
      if (pending_r) mbar_wait(r_full, qc & 1, &never);
    }
  } else if (warp == 1) {
    {
      // ------------------------------------------------------------------ MMA issuer
      // The whole warp runs the loop with warp-uniform descriptors and one elected lane issues each MMA / commit
      // (measured 6 % faster on the sparse configuration-3 backward than a lane-0 loop).
      auto wait_ = [&](uint32_t bar, uint32_t parity) -> bool { return warp_wait(bar, parity, abort_flag); };
      auto issue_ = [&](auto&& fn) {
        if (elect_one_sync()) fn();
        __syncwarp();
      };
      constexpr uint32_t kIdescAcc = instr_desc(F32, 128, D, false, true);
      // 3xTF32: each product is hi*hi + hi*lo + lo*hi (the lo*lo term is below fp32 precision).
      constexpr int kPasses = X3 ? 3 : 1;
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
        const int nch = (n_sub + CH - 1) / CH;
        if (nch == 0) continue;
        if (!(ok = wait_(X3 ? r_ready : r_full, qc & 1))) break;
        const uint32_t g0 = g;
        // S (and dP) of chunk c: S = R0 C0^T at TMEM column 0, dP = R1 C1^T at column 64 (both K-major).
        auto issue_sd = [&](int c) -> bool {
          const uint32_t gg = g0 + c;
          const int st = gg % C::NS;
          const int n_in = min(CH, n_sub - CH * c);
          const int sdb = gg % C::NSD;
          if (!wait_(X3 ? c_ready(st) : c_full(st), (gg / C::NS) & 1)) return false;
          if constexpr (C::G_TMEM) {
            if (!wait_(g_empty(sdb), ((gg / C::NSD) & 1) ^ 1)) return false;
          } else {
            if (!wait_(sd_empty, (gg & 1) ^ 1)) return false;
          }
          tc_fence_after();
          const uint32_t sd_col = C::G_TMEM ? C::SD0 + C::SD_STRIDE * sdb : 0;
          const uint32_t idesc = instr_desc(F32, 128, 32 * n_in, false, false);
          const uint32_t sb = stage(st);
  #pragma unroll
          for (int op = 0; op < C::NR; ++op) {
            const int cs = op == 0 ? 0 : C::SLOT_C1;
            const uint64_t r_hi = smem_desc(r_op(op, 0), 16, 1024), r_lo = smem_desc(r_op(op, 1), 16, 1024);
            const uint64_t c_hi = smem_desc(slot(sb, cs, 0), 16, 1024), c_lo = smem_desc(slot(sb, cs, 1), 16, 1024);
  #pragma unroll
            for (int pass = 0; pass < kPasses; ++pass) {
  #pragma unroll
              for (int kk = 0; kk < D / C::KSTEP; ++kk) {
                const uint32_t cb = kk / 4, within = (kk % 4) * 32;
                const uint64_t a = (pass == 2 ? r_lo : r_hi) + ((cb * C::ROWS * 128 + within) >> 4);
                const uint64_t bd = (pass == 1 ? c_lo : c_hi) + ((cb * C::COLS * 128 + within) >> 4);
                if (op < C::NR_TMEM) {
                  // A = the row operand in TMEM (3xTF32: its lo copy D columns on in the third pass): K = 8 tf32
                  // elements = 8 columns per MMA.
                  const uint32_t a_t = tmem + op * D * C::XL + (pass == 2 ? D : 0) + 8 * kk;
                  issue_([&] { mma_ts<true>(tmem + sd_col + C::DP_OFF * op, a_t, bd, idesc, (pass > 0 || kk > 0) ? 1u : 0u); });
                } else {
                  issue_([&] { mma_ss<F32>(tmem + sd_col + C::DP_OFF * op, a, bd, idesc, (pass > 0 || kk > 0) ? 1u : 0u); });
                }
              }
            }
          }
          issue_([&] {
            mma_commit(C::G_TMEM ? sd_full_b(sdb) : sd_full);
            if (c == nch - 1) mma_commit(r_empty);
          });
          if (lane == 0) FWN_TR(11, c);
          return true;
        };
        // acc0 += dS C0 and / or acc1 += P C1 of chunk c (C0 / C1 as MN-major B operands: the K-major tile
        // itself for bf16, the 32-byte-atom copy for tf32).
        auto issue_acc = [&](int c) -> bool {
          const uint32_t gg = g0 + c;
          const int st = gg % C::NS, gb = gg % C::NB;
          const int n_in = min(CH, n_sub - CH * c);
          if (!wait_(g_full(gb), (gg / C::NB) & 1)) return false;
          if (c == 0 && !wait_(acc_empty, (qc & 1) ^ 1)) return false;
          tc_fence_after();
          const uint32_t sb = stage(st);
          const int ksteps = n_in * C::SUB / C::KSTEP;
  #pragma unroll
          for (int which = 0; which < 2; ++which) {
            if (which == 0 && !C::ACC_DS) continue;
            if (which == 1 && !C::ACC_P) continue;
            const int bs = which == 0 ? (F32 ? C::SLOT_C0MN : 0) : (F32 ? C::SLOT_C1MN : C::SLOT_C1);
            const int gi = which == 0 ? G_DS : G_P;
            const uint32_t acc = tmem + (which == 0 ? C::ACC0 : C::ACC1);
            if constexpr (C::G_TMEM) {
              // dS (over dP) / P (over S) from TMEM: K = 16 columns per MMA = 8 TMEM columns of packed pairs.
              // K = 16 bf16 (8 columns of pairs) or 8 tf32 (8 columns) per MMA.
              // 3xTF32: G hi (over S) and lo (over dP); hi*hi + hi*lo + lo*hi.
              const uint32_t g_col = tmem + C::SD0 + C::SD_STRIDE * gb;
              const uint64_t b_hi = F32 ? smem_desc(slot(sb, bs, 0), C::COLS * 128, 512, kLayoutSW128Base32B)
                                        : smem_desc(slot(sb, bs, 0), C::COLS * 128, 1024);
              const uint64_t b_lo = smem_desc(slot(sb, bs, 1), C::COLS * 128, 512, kLayoutSW128Base32B);
              for (int pass = 0; pass < kPasses; ++pass) {
                const uint32_t a_col = g_col + (X3 ? (pass == 2 ? C::DP_OFF : 0) : (which == 0 ? C::DP_OFF : 0));
                const uint64_t b_desc = pass == 1 ? b_lo : b_hi;
                for (int kk = 0; kk < ksteps; ++kk)
                  issue_([&] {
                    mma_ts<F32>(acc, a_col + 8 * kk, b_desc + ((kk * C::KSTEP * 128) >> 4), kIdescAcc,
                                (c == 0 && pass == 0 && kk == 0) ? 0u : 1u);
                  });
              }
              continue;
            }
            const uint64_t g_hi = C::G64 ? smem_desc(g_tile(gb, gi, 0), 16, 512, kLayoutSW64) : smem_desc(g_tile(gb, gi, 0), 16, 1024);
            const uint64_t g_lo = C::G64 ? smem_desc(g_tile(gb, gi, 1), 16, 512, kLayoutSW64) : smem_desc(g_tile(gb, gi, 1), 16, 1024);
            const uint64_t b_hi = F32 ? smem_desc(slot(sb, bs, 0), C::COLS * 128, 512, kLayoutSW128Base32B)
                                      : smem_desc(slot(sb, bs, 0), C::COLS * 128, 1024);
            const uint64_t b_lo = F32 ? smem_desc(slot(sb, bs, 1), C::COLS * 128, 512, kLayoutSW128Base32B)
                                      : smem_desc(slot(sb, bs, 1), C::COLS * 128, 1024);
            for (int pass = 0; pass < kPasses; ++pass) {
              for (int kk = 0; kk < ksteps; ++kk) {
                const uint32_t cb = kk / 4, within = (kk % 4) * 32;
                const uint32_t aoff = C::G64 ? kk * 32 : cb * C::ROWS * 128 + within;
                const uint64_t a = (pass == 2 ? g_lo : g_hi) + (aoff >> 4);
                const uint64_t bd = (pass == 1 ? b_lo : b_hi) + ((kk * C::KSTEP * 128) >> 4);
                issue_([&] { mma_ss<F32>(acc, a, bd, kIdescAcc, (c == 0 && pass == 0 && kk == 0) ? 0u : 1u); });
              }
            }
          }
          issue_([&] {
            mma_commit(g_empty(gb));
            mma_commit(c_empty(st));
            if (c == nch - 1) mma_commit(acc_full);
          });
          if (lane == 0) FWN_TR(12, c);
          return true;
        };
        if constexpr (C::NS >= 2 && C::NSD >= 2) {
          // S / dP of chunk c+1 go ahead of the accumulating MMAs of chunk c (two stages in flight).
          for (int c = 0; c <= nch && ok; ++c) {
            if (c < nch && !(ok = issue_sd(c))) break;
            if (c >= 1 && !(ok = issue_acc(c - 1))) break;
          }
        } else {
          // One stage, or one S / dP buffer (QUAD): the accumulating MMAs of chunk c free it before chunk c+1 can
          // land; the other CTAs of the SM fill the tensor pipe meanwhile.
          for (int c = 0; c < nch && ok; ++c) {
            if (!(ok = issue_sd(c))) break;
            if (!(ok = issue_acc(c))) break;
          }
        }
        g = g0 + nch;
        ++qc;
      }
      issue_([&] { mma_commit(drain); });
      volatile int never = 0;
      mbar_wait(drain, 0, &never);
    }
  } else if (X3 && warp >= 6) {
    // ------------------------------------------------------------------ 3xTF32 converter (warps 6-9)
    const int ctid = threadIdx.x - 192;
    uint32_t g = 0, qc = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.n_items && ok; it += gridDim.x) {
      const int pb = it % per_bh;
      const int n_sub = p.ptr2[pb + 1] - p.ptr2[pb];
      const int nch = (n_sub + CH - 1) / CH;
      if (nch == 0) continue;
      if (!(ok = mbar_wait(r_full, qc & 1, abort_flag))) break;
      for (int op = C::NR_TMEM; op < C::NR; ++op) split_tf32(r_op(op, 0), r_op(op, 1), C::R_BYTES, ctid, 128);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(r_ready);
      for (int c = 0; c < nch; ++c, ++g) {
        const int st = g % C::NS;
        if (!(ok = mbar_wait(c_full(st), (g / C::NS) & 1, abort_flag))) break;
        const uint32_t sb = stage(st);
        for (int s = 0; s < C::NC; ++s) split_tf32(slot(sb, s, 0), slot(sb, s, 1), C::C_BYTES, ctid, 128);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(c_ready(st));
      }
      ++qc;
    }
  } else {
    // ------------------------------------------------------------------ elementwise + epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    constexpr float kLog2e = 1.4426950408889634f;
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
      const int nch = (n_sub + CH - 1) / CH;
      const int grow = pb * C::ROWS + row;
      float lse2_row = 0.f, delta_row = 0.f;
      if (!C::ROWS_ARE_KEYS) {
        lse2_row = p.lse[static_cast<size_t>(bh) * p.lse_rows + grow] * kLog2e;
        delta_row = p.delta[static_cast<size_t>(bh) * p.lse_rows + grow];
      }
      if constexpr (C::R_TMEM) {
        // The item's row operands into TMEM (this thread's row into its lane), once the previous item's last S / dP
        // MMA is complete; rows past n are zero (as the TMA loads' out-of-range fill).
        if (nch > 0) {
          if (!(ok = mbar_wait(r_empty, (qc & 1) ^ 1, abort_flag))) break;
          tc_fence_after();
#pragma unroll
          for (int op = 0; op < C::NR_TMEM; ++op) {
            const float* src = nullptr;
            if (grow < p.n) {
              src = static_cast<const float*>(op == 0 ? p.r0 : p.r1) +
                    (op == 0 ? static_cast<int64_t>(b) * p.r0_sb + static_cast<int64_t>(grow) * p.r0_sn +
                                   static_cast<int64_t>(h) * p.r0_sh
                             : static_cast<int64_t>(b) * p.r1_sb + static_cast<int64_t>(grow) * p.r1_sn +
                                   static_cast<int64_t>(h) * p.r1_sh);
            }
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
                tmem_st32(trow + op * D * C::XL + D + 32 * j, lo);
              }
              tmem_st32(trow + op * D * C::XL + 32 * j, v);
            }
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(r_full);
        }
      }
      const uint32_t g0 = g;
      for (int c = 0; c < nch; ++c) {
        const uint32_t gg = g0 + c;
        const int st = gg % C::NS, gb = gg % C::NB;
        const int n_in = min(CH, n_sub - CH * c);
        // bf16: S / dP buffer gb (= gg % NSD), whose columns take dS / P; tf32: the one S / dP buffer and
        // shared-memory dS / P buffer gb.
        if (!(ok = mbar_wait(C::G_TMEM ? sd_full_b(gb) : sd_full, C::G_TMEM ? (gg / C::NB) & 1 : gg & 1, abort_flag))) break;
        if (lane == 0) FWN_TR(20, c);
        if (!(ok = mbar_wait(c_full(st), (gg / C::NS) & 1, abort_flag))) break;
        if (!C::G_TMEM && !(ok = mbar_wait(g_empty(gb), ((gg / C::NB) & 1) ^ 1, abort_flag))) break;
        if (lane == 0) FWN_TR(29, c);
        tc_fence_after();
        const uint32_t sb = stage(st);
        const uint32_t sd_col = C::G_TMEM ? C::SD0 + C::SD_STRIDE * gb : 0;
        // One 32-column tile at a time: S and dP of the tile from TMEM, P and dS into TMEM over them (bf16) or into
        // the shared-memory tiles of buffer gb (tf32: TMEM is released once the last tile's values are in registers).
#pragma unroll
        if constexpr (C::QUAD) {
          // Four CTAs per SM leave 80 registers: the tile's 32 columns in two halves of 16 (S and dP of a half from
          // TMEM, its dS pairs over the half's first 8 dP columns, which the other half does not read), so that no
          // thread holds 64 values at once (the one-pass form spilled 76 bytes per thread; this one takes 68 registers
          // and made the dQ pass 10 % faster at configuration 3, results bit-identical).
          const uint32_t w_all = ld_shared_u32(sb + C::BITS_OFF + row * 4);
          const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf) {
            float s[16], dp[16];
            tmem_ld16(trow + sd_col + 16 * hf, s);
            tmem_ld16(trow + sd_col + C::DP_OFF + 16 * hf, dp);
            tmem_wait_ld();
            reg_fence(s);
            reg_fence(dp);
            const uint32_t w = w_all >> (16 * hf);
            const uint32_t any = __reduce_or_sync(0xffffffffu, w & 0xFFFFu);
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              if ((any >> (8 * g)) & 0xFFu) {
#pragma unroll
                for (int ii = 0; ii < 8; ii += 2) {
                  const int i = 8 * g + ii;
                  const float2 x = ffma2(make_float2(s[i], s[i + 1]), sc2, make_float2(-lse2_row, -lse2_row));
                  const float e0 = ex2(x.x), e1 = ex2(x.y);
                  const float p0 = (w & (1u << i)) ? e0 : 0.f, p1 = (w & (1u << (i + 1))) ? e1 : 0.f;
                  const float2 ds = fmul2(make_float2(p0, p1),
                                          fsub2(make_float2(dp[i], dp[i + 1]), make_float2(delta_row, delta_row)));
                  dp[i] = ds.x;
                  dp[i + 1] = ds.y;
                }
              } else {
#pragma unroll
                for (int ii = 0; ii < 8; ++ii) dp[8 * g + ii] = 0.f;
              }
            }
            uint32_t pk[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) pk[i] = pack_bf16(dp[2 * i], dp[2 * i + 1]);
            tmem_st8(trow + sd_col + C::DP_OFF + 8 * hf, pk);
          }
        } else
        for (int j = 0; j < CH; ++j) {
          if (j < n_in) {
            float s[32], dp[32];
            tmem_ld32(trow + sd_col + 32 * j, s);
            if constexpr (C::NEED_DP) tmem_ld32(trow + sd_col + C::DP_OFF + 32 * j, dp);
            const uint32_t w = ld_shared_u32(sb + C::BITS_OFF + j * 512 + row * 4);  // while S / dP are read
            tmem_wait_ld();
            reg_fence(s);
            if constexpr (C::NEED_DP) reg_fence(dp);
            if (!C::G_TMEM && j == n_in - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(sd_empty);
            }
            const uint32_t any = __reduce_or_sync(0xffffffffu, w);
            const float2 sc2 = make_float2(p.scale_log2, p.scale_log2);
            // Groups of 8 columns that no row of the warp may attend to are skipped by the whole warp. Column
            // pairs in f32x2 arithmetic; the columns' lse (log2 units, see the producer) and delta (rows are
            // keys) as broadcast 16-byte shared-memory loads.
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              if ((any >> (8 * g)) & 0xFFu) {
                float l2v[8], dlv[8];
                if constexpr (C::ROWS_ARE_KEYS) {
                  const uint32_t va = sb + C::VEC_OFF + j * 256 + g * 32;
                  const float4 a0 = ld_shared_f32x4(va), a1 = ld_shared_f32x4(va + 16);
                  const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
                  for (int ii = 0; ii < 8; ++ii) l2v[ii] = GATHER ? av[ii] : av[ii] * kLog2e;
                  if constexpr (C::NEED_DP) {
                    const float4 d0 = ld_shared_f32x4(va + 128), d1 = ld_shared_f32x4(va + 144);
                    const float dv[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
                    for (int ii = 0; ii < 8; ++ii) dlv[ii] = dv[ii];
                  }
                } else {
#pragma unroll
                  for (int ii = 0; ii < 8; ++ii) {
                    l2v[ii] = lse2_row;
                    dlv[ii] = delta_row;
                  }
                }
#pragma unroll
                for (int ii = 0; ii < 8; ii += 2) {
                  const int i = 8 * g + ii;
                  const float2 x = ffma2(make_float2(s[i], s[i + 1]), sc2, make_float2(-l2v[ii], -l2v[ii + 1]));
                  const float e0 = ex2(x.x), e1 = ex2(x.y);
                  const float p0 = (w & (1u << i)) ? e0 : 0.f, p1 = (w & (1u << (i + 1))) ? e1 : 0.f;
                  s[i] = p0;
                  s[i + 1] = p1;
                  if constexpr (C::NEED_DP) {
                    const float2 ds = fmul2(make_float2(p0, p1),
                                            fsub2(make_float2(dp[i], dp[i + 1]), make_float2(dlv[ii], dlv[ii + 1])));
                    dp[i] = ds.x;
                    dp[i + 1] = ds.y;
                  }
                }
              } else {
#pragma unroll
                for (int ii = 0; ii < 8; ++ii) {
                  s[8 * g + ii] = 0.f;
                  if constexpr (C::NEED_DP) dp[8 * g + ii] = 0.f;
                }
              }
            }
#pragma unroll
            for (int which = 0; which < 2; ++which) {
              if (which == 0 && !C::ACC_DS) continue;
              if (which == 1 && !C::ACC_P) continue;
              const float* src = which == 0 ? dp : s;
              const uint32_t base = g_tile(gb, which == 0 ? G_DS : G_P, 0);
              if constexpr (C::G_TMEM && X3) {
                // hi (13 low mantissa bits cleared) over S, lo = x - hi over dP.
                float hv[32], lv[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                  hv[i] = __uint_as_float(__float_as_uint(src[i]) & 0xFFFFE000u);
                  lv[i] = src[i] - hv[i];
                }
                tmem_st32(trow + sd_col + C::GW * j, hv);
                tmem_st32(trow + sd_col + C::DP_OFF + C::GW * j, lv);
              } else if constexpr (C::G_TMEM && F32) {
                // 32 fp32 columns over S (P) or dP (dS).
                tmem_st32(trow + sd_col + (which == 0 ? C::DP_OFF : 0) + C::GW * j,
                          *reinterpret_cast<const float(*)[32]>(src));
              } else if constexpr (C::G_TMEM) {
                // 32 bf16 columns = 16 TMEM columns of packed pairs over the first half of S (P) or dP (dS).
                uint32_t pk[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) pk[i] = pack_bf16(src[2 * i], src[2 * i + 1]);
                tmem_st16(trow + sd_col + (which == 0 ? C::DP_OFF : 0) + C::GW * j, pk);
              } else if constexpr (C::G64) {
                // 32 bf16 columns = one 64-byte row.
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                  st_shared_v4(base + sw64_offset(row, cc), pack_bf16(src[8 * cc], src[8 * cc + 1]),
                               pack_bf16(src[8 * cc + 2], src[8 * cc + 3]), pack_bf16(src[8 * cc + 4], src[8 * cc + 5]),
                               pack_bf16(src[8 * cc + 6], src[8 * cc + 7]));
              } else if constexpr (!F32) {
                // 32 bf16 columns = chunks 4j .. 4j+3 of the 128-byte row.
#pragma unroll
                for (int cc = 0; cc < 4; ++cc)
                  st_shared_v4(base + sw128_offset(row, 4 * j + cc), pack_bf16(src[8 * cc], src[8 * cc + 1]),
                               pack_bf16(src[8 * cc + 2], src[8 * cc + 3]), pack_bf16(src[8 * cc + 4], src[8 * cc + 5]),
                               pack_bf16(src[8 * cc + 6], src[8 * cc + 7]));
              } else if constexpr (X3) {
                // hi (13 low mantissa bits cleared) and lo = x - hi tiles.
                const uint32_t lo_base = g_tile(gb, which == 0 ? G_DS : G_P, 1);
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                  uint32_t hv[4], lv[4];
#pragma unroll
                  for (int i = 0; i < 4; ++i) {
                    hv[i] = __float_as_uint(src[4 * cc + i]) & 0xFFFFE000u;
                    lv[i] = __float_as_uint(src[4 * cc + i] - __uint_as_float(hv[i]));
                  }
                  const uint32_t off = j * C::ROWS * 128 + sw128_offset(row, cc);
                  st_shared_v4(base + off, hv[0], hv[1], hv[2], hv[3]);
                  st_shared_v4(lo_base + off, lv[0], lv[1], lv[2], lv[3]);
                }
              } else {
                // 32 fp32 columns = one whole 128-byte column block.
#pragma unroll
                for (int cc = 0; cc < 8; ++cc)
                  st_shared_v4(base + j * C::ROWS * 128 + sw128_offset(row, cc), __float_as_uint(src[4 * cc]),
                               __float_as_uint(src[4 * cc + 1]), __float_as_uint(src[4 * cc + 2]),
                               __float_as_uint(src[4 * cc + 3]));
              }
            }
          }
        }
        if constexpr (C::G_TMEM) {
          tmem_wait_st();
        } else {
          fence_proxy_async_smem();  // shared-memory dS / P -> tensor core reads
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(g_full(gb));
        if (lane == 0) FWN_TR(21, c);
      }
      if (!ok) break;
      g = g0 + nch;
      // ---------------------------------------------------------------- epilogue
      const bool store = grow < p.n;
      const int64_t roff = (static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(grow) * p.o_sn +
                            static_cast<int64_t>(h) * p.o_sh) * C::ES;
      uint8_t* dst0 = C::ACC_DS ? reinterpret_cast<uint8_t*>(p.out0) + roff : nullptr;
      uint8_t* dst1 = C::ACC_P ? reinterpret_cast<uint8_t*>(p.out1) + roff : nullptr;
      if (nch == 0) {
        if (store) {
          if (C::ACC_DS)
            for (int i = 0; i < D * C::ES / 16; ++i) reinterpret_cast<uint4*>(dst0)[i] = make_uint4(0, 0, 0, 0);
          if (C::ACC_P)
            for (int i = 0; i < D * C::ES / 16; ++i) reinterpret_cast<uint4*>(dst1)[i] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      if (!(ok = mbar_wait(acc_full, qc & 1, abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int which = 0; which < 2; ++which) {
        if (which == 0 && !C::ACC_DS) continue;
        if (which == 1 && !C::ACC_P) continue;
        uint8_t* dst = which == 0 ? dst0 : dst1;
        const float mul = which == 0 ? p.scale : 1.f;
        const uint32_t col = which == 0 ? C::ACC0 : C::ACC1;
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
          float o[32];
          tmem_ld32(trow + col + 32 * j, o);
          tmem_wait_ld();
          if (store) {
            if constexpr (!F32) {
#pragma unroll
              for (int i = 0; i < 4; ++i)
                reinterpret_cast<uint4*>(dst + j * 64)[i] =
                    make_uint4(pack_bf16(o[8 * i] * mul, o[8 * i + 1] * mul), pack_bf16(o[8 * i + 2] * mul, o[8 * i + 3] * mul),
                               pack_bf16(o[8 * i + 4] * mul, o[8 * i + 5] * mul), pack_bf16(o[8 * i + 6] * mul, o[8 * i + 7] * mul));
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i)
                reinterpret_cast<float4*>(dst + j * 128)[i] =
                    make_float4(o[4 * i] * mul, o[4 * i + 1] * mul, o[4 * i + 2] * mul, o[4 * i + 3] * mul);
            }
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
