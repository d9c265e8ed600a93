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
__global__ void __launch_bounds__(256) cond_layernorm_kernel(float* __restrict__ x, int64_t rows, int rows_per_sample,
                                                              const int32_t* __restrict__ out_node,
                                                              const float* __restrict__ scale_offset, float eps,
                                                              void* __restrict__ out,
                                                              const __nv_bfloat16* __restrict__ residual) {
  constexpr int V = D / 128;  // float4 per lane
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps leave together (rows are warp-uniform)
  float4* xr = reinterpret_cast<float4*>(x + row * D);
  float4 v[V];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    if constexpr (RES) {
      // x += residual (4 bf16 per lane and step), written back to the residual stream.
      v[i] = xr[lane + 32 * i];
      const uint2 r = __ldg(reinterpret_cast<const uint2*>(residual + row * D) + lane + 32 * i);
      const float2 r01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.x));
      const float2 r23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&r.y));
      v[i].x += r01.x;
      v[i].y += r01.y;
      v[i].z += r23.x;
      v[i].w += r23.y;
      xr[lane + 32 * i] = v[i];
    } else {
      v[i] = __ldg(xr + lane + 32 * i);
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
cudaError_t launch(float* x, int64_t rows, int rows_per_sample, const int32_t* out_node, const float* so, float eps,
                   void* out, bool bf16_out, const __nv_bfloat16* residual, cudaStream_t stream) {
  const int64_t threads = rows * 32;
  const unsigned grid = static_cast<unsigned>((threads + 255) / 256);
  if (bf16_out)
    cond_layernorm_kernel<D, true, RES><<<grid, 256, 0, stream>>>(x, rows, rows_per_sample, out_node, so, eps, out,
                                                                  residual);
  else
    cond_layernorm_kernel<D, false, RES><<<grid, 256, 0, stream>>>(x, rows, rows_per_sample, out_node, so, eps, out,
                                                                   residual);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_d(float* x, int64_t rows, int rows_per_sample, const int32_t* out_node, const float* so, float eps,
                     void* out, bool bf16_out, const __nv_bfloat16* residual, cudaStream_t stream) {
  return residual ? launch<D, true>(x, rows, rows_per_sample, out_node, so, eps, out, bf16_out, residual, stream)
                  : launch<D, false>(x, rows, rows_per_sample, out_node, so, eps, out, bf16_out, residual, stream);
}

}  // namespace

cudaError_t launch_cond_layernorm(float* x, int64_t rows, int d, int rows_per_sample, const int32_t* out_node,
                                  const float* so, float eps, void* out, bool bf16_out, const void* residual,
                                  cudaStream_t stream) {
  if (rows == 0) return cudaSuccess;
  const auto* res = static_cast<const __nv_bfloat16*>(residual);
  switch (d) {
    case 128: return launch_d<128>(x, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    case 256: return launch_d<256>(x, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    case 512: return launch_d<512>(x, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    case 1024: return launch_d<1024>(x, rows, rows_per_sample, out_node, so, eps, out, bf16_out, res, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fwn
