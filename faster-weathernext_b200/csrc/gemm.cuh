// Dense bf16 GEMM with a fused bias / GELU epilogue for the processor's projections around the attention
// (src/faster_weathernext/patch.py:165-177, 250-252: q / k / v projection, mha_final, the MLP):
//   C[m, n] = act(A[m, k] B[k, n] + bias[n]),  A row-major [m, k], B given transposed as Bt [n, k] (both operands
//   K-major), C row-major [m, n] bf16, float32 accumulation, act = identity or GELU in its tanh form.
//
// Persistent, one CTA per SM, tiles of 128 x 256 walked in (row block, column block) order so that the CTAs working
// at the same time share their A rows in L2 (B, a weight, stays in L2):
//   warp 0      TMA producer: A box 64 x 128 and Bt box 64 x 256 (128-byte swizzle) per K-step of 64, into a
//               ring of four 48 KB stages;
//   warp 1      MMA issuer: four tcgen05.mma (M 128, N 256, K 16) per stage into one of two TMEM accumulators
//               (256 columns each), committing the stage back to the producer and, after the tile's last stage,
//               the accumulator to the epilogue;
//   warps 2-9   epilogue: warps w and w+4 share TMEM lane quadrant w % 4 (rows) and take 128 columns each; they
//               read the accumulator in 64-column steps and release it after the last, so the next tile's MMAs
//               (into the other accumulator, then this one) overlap the activation and stores; bias, activation,
//               bf16; each warp's 32 x 32 chunk goes through its own shared-memory buffer (64-byte swizzle, two
//               per warp) and leaves as one TMA tensor store (rows past m clipped by the tensor map). For the
//               training path's MLP two more epilogues: GELU that also stores its input (the pre-activation the
//               backward needs) through a second tensor map, and x GELU'(pre) (the GELU backward fused into the
//               GEMM that produces the gradient of the activation).
// Measured at m = 655,392, k = 512 (n = 1536): stores of one row per lane straight from registers (32 rows per warp
// instruction) held the kernel at 0.82 PFLOP/s; 256 x 256 tiles with each 128-row half single-buffered in TMEM made
// the next tile's MMAs wait for most of the epilogue (1.03 with per-warp TMA stores).
// Every wait is bounded (mbar_wait); on expiry the CTA's roles leave their loops and the CTA frees TMEM.
#pragma once

#include "common.cuh"

namespace fwn {

struct GemmParams {
  const __nv_bfloat16* bias;    // [n] or null
  __nv_bfloat16* c;             // [m, n]
  const __nv_bfloat16* aux_in;  // act 4: the pre-activation [m, n] the GELU was applied to
  // act 5: rows added before the activation, c[i] = act(a b + bias + add0[idx0[i]] + add1[idx1[i]]); an add tensor
  // may be null, an index null (row i itself); rows0 / rows1 bound the indices.
  const __nv_bfloat16* add0;
  const int32_t* idx0;
  const __nv_bfloat16* add1;
  const int32_t* idx1;
  int64_t rows0, rows1;
  int swish;                    // act 5: swish (x sigmoid(x)) after the adds, else identity
  int64_t m;
  int n, k;
  int act;                      // 0 identity, 1 GELU (tanh form), 3 GELU and x itself to the aux output (tm_aux),
                                // 4 x GELU'(aux_in): the backward of GELU, x the incoming gradient, 5 gathered adds
                                // and optional swish (the interaction network's edge and node MLP input layers)
  int n_tiles, num_tiles;
};

// ACT 4 (the GELU backward) fetches its pre-activation tile by TMA into the epilogue warps' staging buffers: three
// stages and four 2 KB buffers per warp (its tile's four 32 x 32 chunks), plus one barrier per epilogue warp.
template <int ACT>
struct GemmCfgT {
  static constexpr int BM = 128, BN = 256, BK = 64;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int NS = ACT == 4 ? 3 : 4;
  static constexpr int NBUF = ACT == 4 ? 4 : 2;                       // staging buffers per epilogue warp
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int THREADS = 320;
  static constexpr int N_BAR = 2 * NS + 4 + 1 + (ACT == 4 ? 8 : 0);
  static constexpr int OUT_BYTES = 32 * 32 * 2;                        // one epilogue warp's 32 x 32 chunk
  static constexpr int OFF_OUT = NS * STAGE_BYTES;                     // 8 warps x NBUF buffers
  static constexpr int OFF_BAR = OFF_OUT + 8 * NBUF * OUT_BYTES;
  static constexpr int SMEM_BYTES = OFF_BAR + N_BAR * 8 + 16 + 1024;  // + TMEM holder / abort word + 1 KB alignment
  static_assert(A_BYTES % 1024 == 0 && B_BYTES % 1024 == 0, "1 KB-aligned stages");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};
using GemmCfg = GemmCfgT<0>;

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// Box {32 columns, 32 rows} of the output from shared memory (bulk async-group completion).
__device__ __forceinline__ void tma_store_2d(const void* tmap, int c0, int c1, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// GELU, tanh form: 0.5 x (1 + tanh(sqrt(2 / pi) (x + 0.044715 x^3))).
__device__ __forceinline__ float gelu_tanh(float x) {
  const float u = 0.7978845608028654f * fmaf(0.044715f * x, x * x, x);
  return 0.5f * x * (1.f + tanh_approx(u));
}

// swish(x) = x sigmoid(x) = 0.5 x + 0.5 x tanh(x / 2): one hardware tanh and two FMAs (x / (1 + exp(-x)) costs an
// exponential and a full-precision division per element, which made the epilogue the GEMM's bottleneck).
__device__ __forceinline__ float swish(float x) {
  const float h = 0.5f * x;
  return fmaf(h, tanh_approx(h), h);
}

// d/dx of the tanh-form GELU: 0.5 (1 + t) + 0.5 x (1 - t^2) sqrt(2 / pi) (1 + 3 * 0.044715 x^2), t = tanh(u).
__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float x2 = x * x;
  const float t = tanh_approx(0.7978845608028654f * fmaf(0.044715f * x, x2, x));
  const float du = 0.7978845608028654f * fmaf(3.f * 0.044715f, x2, 1.f);
  return fmaf(0.5f * x * du, fmaf(-t, t, 1.f), 0.5f * (1.f + t));
}

// Ten warps: each SM sub-partition holds three, which leaves 168 registers per thread. ACT is the epilogue
// (GemmParams::act), a template parameter so that each instantiation carries only its own epilogue code (a runtime
// switch between the four cost the plain GELU epilogue 40 % at the processor's shapes).
template <int ACT>
__global__ void __maxnreg__(168)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_c, const __grid_constant__ CUtensorMap tm_aux,
                     const GemmParams p) {
  using C = GemmCfgT<ACT>;
  extern __shared__ uint8_t smem_gemm[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_gemm) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  auto a_st = [&](int s) { return sbase + s * C::STAGE_BYTES; };
  auto b_st = [&](int s) { return sbase + s * C::STAGE_BYTES + C::A_BYTES; };
  const uint32_t bar0 = sbase + C::OFF_BAR;
  auto full = [&](int s) { return bar0 + 8 * s; };
  auto empty = [&](int s) { return bar0 + 8 * (C::NS + s); };
  auto acc_full = [&](int b) { return bar0 + 8 * (2 * C::NS + b); };
  auto acc_empty = [&](int b) { return bar0 + 8 * (2 * C::NS + 2 + b); };
  const uint32_t drain = bar0 + 8 * (2 * C::NS + 4);
  auto aux_bar = [&](int w) { return bar0 + 8 * (2 * C::NS + 5 + w); };  // ACT 4: epilogue warp w's chunk loads
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + C::OFF_BAR + C::N_BAR * 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::OFF_BAR + C::N_BAR * 8 + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = p.k / C::BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::NS; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);
    }
    mbar_init(drain, 1);
    if constexpr (ACT == 4)
      for (int w = 0; w < 8; ++w) mbar_init(aux_bar(w), 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
    tma_prefetch_desc(&tm_c);
    if (ACT == 3) tma_prefetch_desc(&tm_aux);
  }
  if (warp == 1) tmem_alloc(smem_u32(tmem_holder), C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    uint32_t g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int st = g % C::NS;
        if (!(ok = mbar_wait(empty(st), ((g / C::NS) & 1) ^ 1, abort_flag))) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(full(st), C::STAGE_BYTES);
          tma_load_2d(a_st(st), &tm_a, kb * C::BK, mt * C::BM, full(st));
          tma_load_2d(b_st(st), &tm_b, kb * C::BK, nt * C::BN, full(st));
        }
        __syncwarp();
      }
    }
    if (!ok && lane == 0) {
      // Drain (bounded, ignoring the abort flag): every copy this warp issued lands before TMEM is released.
      volatile int never = 0;
      for (uint32_t k = (g >= C::NS ? g - C::NS : 0); k < g; ++k) mbar_wait(full(k % C::NS), (k / C::NS) & 1, &never);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = instr_desc(false, C::BM, C::BN, false, false);
    uint32_t g = 0, acc_i = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++acc_i) {
      const int buf = acc_i & 1;
      if (!(ok = warp_wait(acc_empty(buf), ((acc_i >> 1) & 1) ^ 1, abort_flag))) break;
      tc_fence_after();
      for (int kb = 0; kb < nk; ++kb, ++g) {
        const int st = g % C::NS;
        if (!(ok = warp_wait(full(st), (g / C::NS) & 1, abort_flag))) break;
        tc_fence_after();
        const uint64_t ad = smem_desc(a_st(st), 16, 1024), bd = smem_desc(b_st(st), 16, 1024);
        if (elect_one_sync()) {
#pragma unroll
          for (int kk = 0; kk < C::BK / 16; ++kk)
            mma_ss<false>(tmem + buf * C::BN, ad + ((kk * 32) >> 4), bd + ((kk * 32) >> 4), idesc,
                          (kb > 0 || kk > 0) ? 1u : 0u);
          mma_commit(empty(st));
          if (kb == nk - 1) mma_commit(acc_full(buf));
        }
        __syncwarp();
      }
    }
    if (elect_one_sync()) mma_commit(drain);
    __syncwarp();
    volatile int never = 0;
    mbar_wait(drain, 0, &never);
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-9)
    const int quarter = warp & 3, half = (warp - 2) >> 2;  // rows 32 quarter + lane, columns 128 half + [0, 128)
    const uint32_t trow = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + half * 128;
    auto out_buf = [&](int b) { return sbase + C::OFF_OUT + ((warp - 2) * C::NBUF + b) * C::OUT_BYTES; };
    uint32_t acc_i = 0, nbuf = 0;
    bool ok = true, aux_pending = false;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, ++acc_i) {
      const int mt = t / p.n_tiles, nt = t % p.n_tiles;
      const int buf = acc_i & 1;
      const int64_t row0 = static_cast<int64_t>(mt) * C::BM + quarter * 32;  // the warp's first row
      const int col0 = nt * C::BN + half * 128;
      if constexpr (ACT == 4) {
        // The pre-activation of this warp's four 32 x 32 chunks into its buffers (rows past m read as 0), once the
        // previous tile's stores have read them; the loads overlap the wait for the accumulator.
        if (lane == 0) {
          bulk_wait_read<0>();
          mbar_arrive_expect_tx(aux_bar(warp - 2), 4 * C::OUT_BYTES);
          for (int q = 0; q < 4; ++q)
            tma_load_2d(out_buf(q), &tm_aux, col0 + 32 * q, static_cast<int>(row0), aux_bar(warp - 2));
        }
        __syncwarp();
        aux_pending = true;
      }
      if (!(ok = mbar_wait(acc_full(buf), (acc_i >> 1) & 1, abort_flag))) break;
      if constexpr (ACT == 4) {
        if (!(ok = mbar_wait(aux_bar(warp - 2), acc_i & 1, abort_flag))) break;
        aux_pending = false;
      }
      tc_fence_after();
      // act 5: this lane's row of each added tensor (its index read once per tile); -1: no row (past m, or no tensor).
      int64_t ar0 = -1, ar1 = -1;
      if constexpr (ACT == 5) {
        const int64_t r = row0 + lane;
        if (r < p.m) {
          if (p.add0 != nullptr) ar0 = p.idx0 != nullptr ? static_cast<int64_t>(__ldg(p.idx0 + r)) : r;
          if (p.add1 != nullptr) ar1 = p.idx1 != nullptr ? static_cast<int64_t>(__ldg(p.idx1 + r)) : r;
          if ((p.add0 != nullptr && static_cast<uint64_t>(ar0) >= static_cast<uint64_t>(p.rows0)) ||
              (p.add1 != nullptr && static_cast<uint64_t>(ar1) >= static_cast<uint64_t>(p.rows1))) {
            // An index outside its tensor: add nothing for this row and report it (fwn_device_error).
            atomicOr(&g_device_error, 0x400u);
            ar0 = ar1 = -1;
          }
        }
      }
#pragma unroll 1
      for (int jp = 0; jp < 2; ++jp) {
        float v[2][32];
        tmem_ld32(trow + buf * C::BN + 64 * jp, v[0]);
        tmem_ld32(trow + buf * C::BN + 64 * jp + 32, v[1]);
        tmem_wait_ld();
        reg_fence(v[0]);
        reg_fence(v[1]);
        if (jp == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty(buf));
        }
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
          const int c32 = col0 + 64 * jp + 32 * jj;
          uint32_t bw[16];  // the chunk's 32 bias values as bf16 pairs (the same 64 bytes for every lane)
          if (p.bias != nullptr) {
            const uint4* bp = reinterpret_cast<const uint4*>(p.bias + c32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w = __ldg(bp + q);
              bw[4 * q] = w.x;
              bw[4 * q + 1] = w.y;
              bw[4 * q + 2] = w.z;
              bw[4 * q + 3] = w.w;
            }
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) bw[i] = 0u;
          }
          uint32_t aw[16];  // act 4: this lane's row of the pre-activation chunk as bf16 pairs (0 past m)
          if constexpr (ACT == 4) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint4 w = ld_shared_u32x4(out_buf(2 * jp + jj) + sw64_offset(lane, q));
              aw[4 * q] = w.x;
              aw[4 * q + 1] = w.y;
              aw[4 * q + 2] = w.z;
              aw[4 * q + 3] = w.w;
            }
          }
          if constexpr (ACT == 5) {
            // The chunk's 32 columns of this lane's rows of the added tensors, into the bias pairs.
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int64_t ar = t == 0 ? ar0 : ar1;
              if (ar < 0) continue;
              const uint4* ap = reinterpret_cast<const uint4*>((t == 0 ? p.add0 : p.add1) + ar * p.n + c32);
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint4 w = __ldg(ap + q);
                const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[e]));
                  v[jj][8 * q + 2 * e] += x.x;
                  v[jj][8 * q + 2 * e + 1] += x.y;
                }
              }
            }
          }
          uint32_t pk[16], px[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float2 bf = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bw[i]));
            float a = v[jj][2 * i] + bf.x, b = v[jj][2 * i + 1] + bf.y;
            if constexpr (ACT == 3) px[i] = pack_bf16(a, b);
            if constexpr (ACT == 1 || ACT == 3) {
              a = gelu_tanh(a);
              b = gelu_tanh(b);
            } else if constexpr (ACT == 4) {
              const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&aw[i]));
              a *= gelu_tanh_grad(x.x);
              b *= gelu_tanh_grad(x.y);
            } else if constexpr (ACT == 5) {
              if (p.swish) {
                a = swish(a);
                b = swish(b);
              }
            }
            pk[i] = pack_bf16(a, b);
          }
          // This lane's row of the chunk into the warp's buffer (64-byte swizzle) once the store that last read the
          // buffer has read it, then one TMA store of the 32 x 32 chunk (act 3: the pre-activation first, through
          // the other buffer).
#pragma unroll
          for (int out = (ACT == 3 ? 0 : 1); out < 2; ++out) {
            // act 4: the chunk's own buffer, whose pre-activation this lane has just read (each lane its own row).
            const uint32_t ob = ACT == 4 ? out_buf(2 * jp + jj) : out_buf(nbuf & 1);
            const uint32_t* src = out == 0 ? px : pk;
            if (ACT != 4 && lane == 0) bulk_wait_read<1>();
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 4; ++q)
              st_shared_v4(ob + sw64_offset(lane, q), src[4 * q], src[4 * q + 1], src[4 * q + 2], src[4 * q + 3]);
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row0 < p.m) {
              tma_store_2d(out == 0 ? &tm_aux : &tm_c, c32, static_cast<int>(row0), ob);
              bulk_commit();
            }
            ++nbuf;
          }
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    if (ACT == 4 && aux_pending && lane == 0) {
      // Left early with chunk loads in flight: wait (bounded, ignoring the abort flag) until they have landed.
      volatile int never = 0;
      mbar_wait(aux_bar(warp - 2), acc_i & 1, &never);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
}

}  // namespace fwn
