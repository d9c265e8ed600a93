// Grid <-> mesh interaction-network pieces of the processor's encoder / decoder (the blocked GNNs of
// src/faster_weathernext/patch.py:347-509, ChunkedDeepGNN), as HBM-bound kernels around the tcgen05 GEMM:
//
//   gather_add_act  h[e, :] = act(E[e, :] + S[snd[e], :] + R[rcv[e], :] + b)   the first layer of an MLP whose input
//                   is (edge, sender, receiver) features, with the layer's matmul applied per node before the gather
//                   (the reference's pre-gather projections, pre_gather_{senders,receivers,edges}_for_edges_fn);
//                   any of S / R may be absent, E may be absent, indices may be absent (identity). bf16 in and out,
//                   float32 arithmetic; act = identity or swish (x sigmoid(x), through the hardware tanh).
//   ln_segment_sum  out[i, :] = norm * sum over e in [seg[i], seg[i+1]) of LN(m[e, :]) (+ residual[i, :])
//                   LayerNorm with scale / offset over the feature row of each message, summed over the receiver's
//                   edges, which are sorted by receiver so that a receiver's messages are one contiguous run
//                   (the reference's sorted segment_sum, indices_are_sorted=True, with its optional normalisation);
//                   with seg = NULL every row is its own segment (a node MLP's output norm). One warp per receiver,
//                   the running sum in registers: deterministic, no atomics. float32 or bf16 out.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace fwn {

namespace {

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// One thread per 8 features of one edge (16-byte loads of each operand row).
__global__ void __launch_bounds__(256) gather_add_act_kernel(const __nv_bfloat16* __restrict__ e_proj,
                                                             const __nv_bfloat16* __restrict__ s_proj,
                                                             const int32_t* __restrict__ snd,
                                                             const __nv_bfloat16* __restrict__ r_proj,
                                                             const int32_t* __restrict__ rcv,
                                                             const __nv_bfloat16* __restrict__ bias, int64_t rows,
                                                             int h, bool swish, __nv_bfloat16* __restrict__ out) {
  const int per_row = h / 8;
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * per_row) return;
  const int64_t e = idx / per_row;
  const int c = static_cast<int>(idx % per_row) * 8;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, v[8];
  if (e_proj) {
    load8(e_proj + e * h + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  if (s_proj) {
    const int64_t s = snd ? __ldg(snd + e) : e;
    load8(s_proj + s * h + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  if (r_proj) {
    const int64_t r = rcv ? __ldg(rcv + e) : e;
    load8(r_proj + r * h + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  if (bias) {
    load8(bias + c, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] += v[i];
  }
  if (swish) {
    // x sigmoid(x) = 0.5 x + 0.5 x tanh(x / 2): one hardware tanh, no division.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float h = 0.5f * acc[i];
      float t;
      asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(h));
      acc[i] = fmaf(h, t, h);
    }
  }
  uint4 o;
  o.x = pack2(acc[0], acc[1]);
  o.y = pack2(acc[2], acc[3]);
  o.z = pack2(acc[4], acc[5]);
  o.w = pack2(acc[6], acc[7]);
  reinterpret_cast<uint4*>(out + e * h + c)[0] = o;
}

// One warp per receiver; F / 256 groups of 8 features per lane.
template <int F, bool BF16_OUT>
__global__ void __launch_bounds__(256) ln_segment_sum_kernel(const __nv_bfloat16* __restrict__ m,
                                                             const int32_t* __restrict__ seg, int64_t n_out,
                                                             const __nv_bfloat16* __restrict__ gamma,
                                                             const __nv_bfloat16* __restrict__ beta, float eps,
                                                             float norm, const float* residual, void* out) {
  // residual and out may be the same rows (a receiver's sum accumulated over edge blocks): plain loads, no restrict.
  constexpr int G = F / 256;  // 16-byte groups per lane
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= n_out) return;  // whole warps
  const int64_t e0 = seg ? __ldg(seg + i) : i, e1 = seg ? __ldg(seg + i + 1) : i + 1;
  float g[G][8], bt[G][8], sum[G][8];
#pragma unroll
  for (int q = 0; q < G; ++q) {
    load8(gamma + (q * 32 + lane) * 8, g[q]);
    load8(beta + (q * 32 + lane) * 8, bt[q]);
#pragma unroll
    for (int k = 0; k < 8; ++k) sum[q][k] = 0.f;
  }
  for (int64_t e = e0; e < e1; ++e) {
    float v[G][8];
    float s1 = 0.f;
#pragma unroll
    for (int q = 0; q < G; ++q) {
      load8(m + e * F + (q * 32 + lane) * 8, v[q]);
#pragma unroll
      for (int k = 0; k < 8; ++k) s1 += v[q][k];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    const float mean = s1 * (1.f / F);
    float s2 = 0.f;
#pragma unroll
    for (int q = 0; q < G; ++q) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float d = v[q][k] - mean;
        s2 += d * d;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float rstd = rsqrtf(s2 * (1.f / F) + eps);
#pragma unroll
    for (int q = 0; q < G; ++q) {
#pragma unroll
      for (int k = 0; k < 8; ++k) sum[q][k] += (v[q][k] - mean) * rstd * g[q][k] + bt[q][k];
    }
  }
  // The residual rows before any store (residual may be out itself: a load may not pass a store that can alias it).
  float4 res[G][2];
  if (residual) {
#pragma unroll
    for (int q = 0; q < G; ++q) {
      const float4* rp = reinterpret_cast<const float4*>(residual + i * F + (q * 32 + lane) * 8);
      res[q][0] = rp[0];
      res[q][1] = rp[1];
    }
  }
#pragma unroll
  for (int q = 0; q < G; ++q) {
    const int c = (q * 32 + lane) * 8;
    float r[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) r[k] = sum[q][k] * norm;
    if (residual) {
      const float4 a = res[q][0], b = res[q][1];
      r[0] += a.x; r[1] += a.y; r[2] += a.z; r[3] += a.w;
      r[4] += b.x; r[5] += b.y; r[6] += b.z; r[7] += b.w;
    }
    if constexpr (BF16_OUT) {
      uint4 o;
      o.x = pack2(r[0], r[1]);
      o.y = pack2(r[2], r[3]);
      o.z = pack2(r[4], r[5]);
      o.w = pack2(r[6], r[7]);
      reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + i * F + c)[0] = o;
    } else {
      float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + i * F + c);
      o[0] = make_float4(r[0], r[1], r[2], r[3]);
      o[1] = make_float4(r[4], r[5], r[6], r[7]);
    }
  }
}

template <int F>
cudaError_t launch_ln(const __nv_bfloat16* m, const int32_t* seg, int64_t n_out, const __nv_bfloat16* gamma,
                      const __nv_bfloat16* beta, float eps, float norm, const float* residual, void* out, bool bf16_out,
                      cudaStream_t stream) {
  const unsigned grid = static_cast<unsigned>((n_out * 32 + 255) / 256);
  if (bf16_out)
    ln_segment_sum_kernel<F, true><<<grid, 256, 0, stream>>>(m, seg, n_out, gamma, beta, eps, norm, residual, out);
  else
    ln_segment_sum_kernel<F, false><<<grid, 256, 0, stream>>>(m, seg, n_out, gamma, beta, eps, norm, residual, out);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gather_add_act(const void* e_proj, const void* s_proj, const int32_t* snd, const void* r_proj,
                                  const int32_t* rcv, const void* bias, int64_t rows, int h, bool swish, void* out,
                                  cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const int64_t threads = rows * (h / 8);
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  gather_add_act_kernel<<<grid, 256, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(e_proj), static_cast<const __nv_bfloat16*>(s_proj), snd,
      static_cast<const __nv_bfloat16*>(r_proj), rcv, static_cast<const __nv_bfloat16*>(bias), rows, h, swish,
      static_cast<__nv_bfloat16*>(out));
  return cudaGetLastError();
}

cudaError_t launch_ln_segment_sum(const void* m, const int32_t* seg, int64_t n_out, int f, const void* gamma,
                                  const void* beta, float eps, float norm, const float* residual, void* out,
                                  bool bf16_out, cudaStream_t stream) {
  if (n_out == 0) return cudaSuccess;
  const auto* mm = static_cast<const __nv_bfloat16*>(m);
  const auto* g = static_cast<const __nv_bfloat16*>(gamma);
  const auto* b = static_cast<const __nv_bfloat16*>(beta);
  switch (f) {
    case 256: return launch_ln<256>(mm, seg, n_out, g, b, eps, norm, residual, out, bf16_out, stream);
    case 512: return launch_ln<512>(mm, seg, n_out, g, b, eps, norm, residual, out, bf16_out, stream);
    case 1024: return launch_ln<1024>(mm, seg, n_out, g, b, eps, norm, residual, out, bf16_out, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fwn
