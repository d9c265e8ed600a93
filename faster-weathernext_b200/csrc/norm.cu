// Conditioned LayerNorm of the mesh-transformer processor's pre-LN blocks (src/faster_weathernext/patch.py:
// 238-252, 288-290: LayerNorm without scale / offset followed by the norm conditioning's per-sample scale and
// offset): y = (x - mean) / sqrt(var + eps) * (1 + scale[s]) + offset[s], x float32 [rows, d], s = row / rows
// per sample, y bf16 or float32. One warp per row, the row in registers (d / 32 values per lane, float4
// loads), two passes over registers for the mean and the variance; HBM-bound (4 d bytes read, 2 d or 4 d
// written per row). With an output node map (the node permutation of the reference's transformer, patch.py:
// 275-276, 291-292, fused into the final norm's store), row r of sample s goes to row s * rows_per_sample +
// out_node[r % rows_per_sample]; a map entry outside [0, rows_per_sample) drops its row (no write). With a residual
// input (bf16 [rows, d], the output of the sub-block before the norm), the kernel first adds it into the float32
// residual stream in place (x += residual, as the pre-LN block's `x = x + f(norm(x))`, patch.py:238-252) and
// normalises the sum: one pass of 4 d + 2 d bytes read and 4 d + 2 d (or 4 d) written per row, instead of a separate
// add (4 d + 2 d read, 4 d written) and the norm (4 d read, 2 d written).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace fwn {

namespace {

template <int D, bool BF16_OUT, bool RES>
__global__ void __launch_bounds__(256) cond_layernorm_kernel(const float* x_in, float* x_out, int64_t rows,
                                                              int rows_per_sample,
                                                              const int32_t* __restrict__ out_node,
                                                              const float* __restrict__ scale_offset, float eps,
                                                              void* __restrict__ out,
                                                              const __nv_bfloat16* __restrict__ residual) {
  // x_out (RES only) may be x_in itself (the residual stream updated in place): every load of the row is issued
  // before the first store (the compiler may not move a load across a store that can alias it), and x_in is read
  // through the read-only path only without a residual.
  constexpr int V = D / 128;  // float4 per lane
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps leave together (rows are warp-uniform)
  const float4* xr = reinterpret_cast<const float4*>(x_in + row * D);
  float4 v[V];
  uint2 r[V];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if constexpr (RES) {
      v[i] = xr[lane + 32 * i];
      r[i] = __ldg(reinterpret_cast<const uint2*>(residual + row * D) + lane + 32 * i);
    } else {
      v[i] = __ldg(xr + lane + 32 * i);
    }
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if constexpr (RES) {
      // x_out = x_in + residual (4 bf16 per lane and step).
      const float2 r01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[i].x));
      const float2 r23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r[i].y));
      v[i].x += r01.x;
      v[i].y += r01.y;
      v[i].z += r23.x;
      v[i].w += r23.y;
      reinterpret_cast<float4*>(x_out + row * D)[lane + 32 * i] = v[i];
    }
    sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float mean = sum * (1.0f / D);
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
    sq += (a * a + b * b) + (c * c + d * d);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  const float rstd = rsqrtf(sq * (1.0f / D) + eps);
  const int64_t sample = row / rows_per_sample;
  const float* so = scale_offset + sample * 2 * D;
  int64_t orow = row;
  if (out_node != nullptr) {
    const int node = __ldg(out_node + (row - sample * rows_per_sample));
    if (node < 0 || node >= rows_per_sample) return;  // not a permutation entry: no write (whole warp)
    orow = sample * rows_per_sample + node;
  }
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int col = 4 * (lane + 32 * i);
    const float4 sc = __ldg(reinterpret_cast<const float4*>(so + col));
    const float4 of = __ldg(reinterpret_cast<const float4*>(so + D + col));
    float4 y;
    y.x = (v[i].x - mean) * rstd * (1.f + sc.x) + of.x;
    y.y = (v[i].y - mean) * rstd * (1.f + sc.y) + of.y;
    y.z = (v[i].z - mean) * rstd * (1.f + sc.z) + of.z;
    y.w = (v[i].w - mean) * rstd * (1.f + sc.w) + of.w;
    if constexpr (BF16_OUT) {
      const __nv_bfloat162 lo = __floats2bfloat162_rn(y.x, y.y), hi = __floats2bfloat162_rn(y.z, y.w);
      uint2 packed;
      packed.x = *reinterpret_cast<const uint32_t*>(&lo);
      packed.y = *reinterpret_cast<const uint32_t*>(&hi);
      reinterpret_cast<uint2*>(static_cast<__nv_bfloat16*>(out) + orow * D)[lane + 32 * i] = packed;
    } else {
      reinterpret_cast<float4*>(static_cast<float*>(out) + orow * D)[lane + 32 * i] = y;
    }
  }
}

template <int D, bool RES>
cudaError_t launch(const float* x, float* x_out, int64_t rows, int rows_per_sample, const int32_t* out_node,
                   const float* so, float eps, void* out, bool bf16_out, const __nv_bfloat16* residual,
                   cudaStream_t stream) {
  const int64_t threads = rows * 32;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  if (bf16_out)
    cond_layernorm_kernel<D, true, RES><<<grid, 256, 0, stream>>>(x, x_out, rows, rows_per_sample, out_node, so, eps,
                                                                  out, residual);
  else
    cond_layernorm_kernel<D, false, RES><<<grid, 256, 0, stream>>>(x, x_out, rows, rows_per_sample, out_node, so, eps,
                                                                   out, residual);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_d(const float* x, float* x_out, int64_t rows, int rows_per_sample, const int32_t* out_node,
                     const float* so, float eps, void* out, bool bf16_out, const __nv_bfloat16* residual,
                     cudaStream_t stream) {
  return residual ? launch<D, true>(x, x_out, rows, rows_per_sample, out_node, so, eps, out, bf16_out, residual, stream)
                  : launch<D, false>(x, x_out, rows, rows_per_sample, out_node, so, eps, out, bf16_out, residual,
                                     stream);
}

// Backward of y = LN(x) (1 + scale[s]) + offset[s] (x the normalised input, i.e. the residual stream after any add):
//   g = dy (1 + scale[s]),  dx = dx_in + rstd (g - mean(g) - xhat mean(g xhat))   (one warp per row)
//   dscale[s, j] = sum over the sample's rows of dy xhat,  doffset[s, j] = sum of dy  (per-CTA column partials: each
//   CTA takes kBwdRows consecutive rows of one sample; reduced per sample by cond_layernorm_part_sum_kernel).
constexpr int kBwdRows = 128;

template <int D, bool DY_BF16>
__global__ void __launch_bounds__(256) cond_layernorm_bwd_kernel(const float* __restrict__ x, int rows_per_sample,
                                                                  int ctas_per_sample,
                                                                  const float* __restrict__ scale_offset, float eps,
                                                                  const void* __restrict__ dy,
                                                                  const float* dx_in,
                                                                  float* dx,
                                                                  __nv_bfloat16* __restrict__ dx_bf16,
                                                                  float* __restrict__ part) {
  constexpr int V = D / 128;
  __shared__ float red[8][2 * D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sample = blockIdx.x / ctas_per_sample, chunk = blockIdx.x % ctas_per_sample;
  const int64_t r0 = static_cast<int64_t>(sample) * rows_per_sample + static_cast<int64_t>(chunk) * kBwdRows;
  const int64_t r1 = static_cast<int64_t>(sample) * rows_per_sample +
                     min(static_cast<int64_t>(chunk + 1) * kBwdRows, static_cast<int64_t>(rows_per_sample));
  float4 sc[V], ds[V], dof[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    sc[i] = __ldg(reinterpret_cast<const float4*>(scale_offset + static_cast<int64_t>(sample) * 2 * D) + lane + 32 * i);
    ds[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    dof[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // A row's loads (x, dy, the incoming gradient) are all issued before any of its stores: dx may be dx_in, and the
  // compiler may not move a load across a store that can alias it, which otherwise serialises the row's memory round
  // trips. xhat and g are recomputed in the last loop instead of kept, to stay within two CTAs' registers per SM.
  for (int64_t row = r0 + warp; row < r1; row += 8) {
    float4 v[V], d[V], a[V];
#pragma unroll
    for (int i = 0; i < V; ++i) {
      v[i] = __ldg(reinterpret_cast<const float4*>(x + row * D) + lane + 32 * i);
      if constexpr (DY_BF16) {
        const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(dy) + row * D) + lane + 32 * i);
        const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
        const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
        d[i] = make_float4(lo.x, lo.y, hi.x, hi.y);
      } else {
        d[i] = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(dy) + row * D) + lane + 32 * i);
      }
      a[i] = dx_in ? reinterpret_cast<const float4*>(dx_in + row * D)[lane + 32 * i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float s1 = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) s1 += (v[i].x + v[i].y) + (v[i].z + v[i].w);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    const float mean = s1 * (1.f / D);
    float s2 = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      v[i] = make_float4(v[i].x - mean, v[i].y - mean, v[i].z - mean, v[i].w - mean);  // centred from here on
      s2 += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    const float rstd = rsqrtf(s2 * (1.f / D) + eps);
    float sg = 0.f, sgx = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 xh = make_float4(v[i].x * rstd, v[i].y * rstd, v[i].z * rstd, v[i].w * rstd);
      const float4 g = make_float4(d[i].x * (1.f + sc[i].x), d[i].y * (1.f + sc[i].y), d[i].z * (1.f + sc[i].z),
                                   d[i].w * (1.f + sc[i].w));
      sg += (g.x + g.y) + (g.z + g.w);
      sgx += (g.x * xh.x + g.y * xh.y) + (g.z * xh.z + g.w * xh.w);
      ds[i].x += d[i].x * xh.x; ds[i].y += d[i].y * xh.y; ds[i].z += d[i].z * xh.z; ds[i].w += d[i].w * xh.w;
      dof[i].x += d[i].x; dof[i].y += d[i].y; dof[i].z += d[i].z; dof[i].w += d[i].w;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sg += __shfl_xor_sync(0xffffffffu, sg, o);
      sgx += __shfl_xor_sync(0xffffffffu, sgx, o);
    }
    const float mg = sg * (1.f / D), mgx = sgx * (1.f / D);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const float4 xh = make_float4(v[i].x * rstd, v[i].y * rstd, v[i].z * rstd, v[i].w * rstd);
      const float4 g = make_float4(d[i].x * (1.f + sc[i].x), d[i].y * (1.f + sc[i].y), d[i].z * (1.f + sc[i].z),
                                   d[i].w * (1.f + sc[i].w));
      float4 r = make_float4(rstd * (g.x - mg - xh.x * mgx), rstd * (g.y - mg - xh.y * mgx),
                             rstd * (g.z - mg - xh.z * mgx), rstd * (g.w - mg - xh.w * mgx));
      r.x += a[i].x; r.y += a[i].y; r.z += a[i].z; r.w += a[i].w;
      reinterpret_cast<float4*>(dx + row * D)[lane + 32 * i] = r;
      if (dx_bf16) {
        const __nv_bfloat162 lo = __floats2bfloat162_rn(r.x, r.y), hi = __floats2bfloat162_rn(r.z, r.w);
        uint2 pk;
        pk.x = *reinterpret_cast<const uint32_t*>(&lo);
        pk.y = *reinterpret_cast<const uint32_t*>(&hi);
        reinterpret_cast<uint2*>(dx_bf16 + row * D)[lane + 32 * i] = pk;
      }
    }
  }
  // Column partials of the CTA: warps' sums through shared memory, one row of 2 D per CTA.
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int c = 4 * (lane + 32 * i);
    red[warp][c] = ds[i].x; red[warp][c + 1] = ds[i].y; red[warp][c + 2] = ds[i].z; red[warp][c + 3] = ds[i].w;
    red[warp][D + c] = dof[i].x; red[warp][D + c + 1] = dof[i].y; red[warp][D + c + 2] = dof[i].z;
    red[warp][D + c + 3] = dof[i].w;
  }
  __syncthreads();
  for (int j = threadIdx.x; j < 2 * D; j += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][j];
    part[static_cast<int64_t>(blockIdx.x) * 2 * D + j] = t;
  }
}

// dso[s, j] = sum over the sample's CTAs of part[cta, j] (fixed order: deterministic).
__global__ void __launch_bounds__(256) cond_layernorm_part_sum_kernel(const float* __restrict__ part, int samples,
                                                                       int ctas_per_sample, int width,
                                                                       float* __restrict__ dso) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(samples) * width) return;
  const int s = static_cast<int>(idx / width), j = static_cast<int>(idx % width);
  float t = 0.f;
  for (int c = 0; c < ctas_per_sample; ++c) t += part[(static_cast<int64_t>(s) * ctas_per_sample + c) * width + j];
  dso[idx] = t;
}

template <int D>
cudaError_t launch_bwd(const float* x, int64_t rows, int rows_per_sample, const float* so, float eps, const void* dy,
                       bool dy_bf16, const float* dx_in, float* dx, __nv_bfloat16* dx_bf16, float* dso, float* part,
                       cudaStream_t stream) {
  const int samples = static_cast<int>(rows / rows_per_sample);
  const int cps = (rows_per_sample + kBwdRows - 1) / kBwdRows;
  const unsigned grid = static_cast<unsigned>(samples * cps);
  if (dy_bf16)
    cond_layernorm_bwd_kernel<D, true><<<grid, 256, 0, stream>>>(x, rows_per_sample, cps, so, eps, dy, dx_in, dx,
                                                                 dx_bf16, part);
  else
    cond_layernorm_bwd_kernel<D, false><<<grid, 256, 0, stream>>>(x, rows_per_sample, cps, so, eps, dy, dx_in, dx,
                                                                  dx_bf16, part);
  const int64_t total = static_cast<int64_t>(samples) * 2 * D;
  cond_layernorm_part_sum_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(part, samples, cps,
                                                                                                 2 * D, dso);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_cond_layernorm(const float* x, float* x_out, int64_t rows, int d, int rows_per_sample,
                                  const int32_t* out_node, const float* so, float eps, void* out, bool bf16_out,
                                  const void* residual, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const auto* res = static_cast<const __nv_bfloat16*>(residual);
  switch (d) {
    case 128: return launch_d<128>(x, x_out, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    case 256: return launch_d<256>(x, x_out, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    case 512: return launch_d<512>(x, x_out, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    case 1024: return launch_d<1024>(x, x_out, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    default: return cudaErrorInvalidValue;
  }
}

size_t cond_layernorm_bwd_workspace(int64_t rows, int d, int rows_per_sample) {
  const int64_t samples = rows / rows_per_sample;
  const int64_t cps = (rows_per_sample + kBwdRows - 1) / kBwdRows;
  return static_cast<size_t>(samples * cps * 2 * d) * sizeof(float);
}

cudaError_t launch_cond_layernorm_bwd(const float* x, int64_t rows, int d, int rows_per_sample, const float* so,
                                      float eps, const void* dy, bool dy_bf16, const float* dx_in, float* dx,
                                      void* dx_bf16, float* dso, void* ws, cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  auto* xb = static_cast<__nv_bfloat16*>(dx_bf16);
  auto* part = static_cast<float*>(ws);
  switch (d) {
    case 128: return launch_bwd<128>(x, rows, rows_per_sample, so, eps, dy, dy_bf16, dx_in, dx, xb, dso, part, stream);
    case 256: return launch_bwd<256>(x, rows, rows_per_sample, so, eps, dy, dy_bf16, dx_in, dx, xb, dso, part, stream);
    case 512: return launch_bwd<512>(x, rows, rows_per_sample, so, eps, dy, dy_bf16, dx_in, dx, xb, dso, part, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fwn
