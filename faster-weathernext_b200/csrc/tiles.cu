// Tile-list builder on the GPU: the CUDA counterpart of build_tile_mask
// (src/faster_weathernext/pallas_attn.py:85-109) and the 128-row pairing the attention kernels walk.
//
// One CTA per query block. The block's key blocks are marked in a shared-memory bitmap (one bit per
// 32-key tile), so "distinct, ascending key blocks" (the reference's sorted np.unique) falls out of
// the bitmap order and a tile's index inside the block is a popcount prefix. Mask words are OR-ed
// into shared memory (or, for blocks with very many tiles, straight into the zeroed output).
#include "tiles.cuh"

namespace fwn {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ void mark(uint32_t* bitmap, int kb) {
  atomicOr(&bitmap[kb >> 5], 1u << (kb & 31));
}

// Exclusive prefix of popcount(bitmap[i]) into prefix[i] for i < words; returns the total.
__device__ int bitmap_prefix(const uint32_t* bitmap, int* prefix, int words, int* scratch) {
  const int tid = threadIdx.x;
  const int per = (words + kThreads - 1) / kThreads;
  const int w0 = min(tid * per, words), w1 = min(w0 + per, words);
  int local = 0;
  for (int i = w0; i < w1; ++i) local += __popc(bitmap[i]);
  // Block exclusive scan of `local`.
  const int lane = tid & 31, warp = tid >> 5;
  int incl = local;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= d) incl += y;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int s = lane < kWarps ? scratch[lane] : 0;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, s, d);
      if (lane >= d) s += y;
    }
    if (lane < kWarps) scratch[lane] = s;  // inclusive per-warp totals
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? scratch[warp - 1] : 0);
  for (int i = w0; i < w1; ++i) {
    prefix[i] = run;
    run += __popc(bitmap[i]);
  }
  const int total = scratch[kWarps - 1];
  __syncthreads();
  return total;
}

__device__ __forceinline__ int rank_of(const uint32_t* bitmap, const int* prefix, int kb) {
  const uint32_t w = bitmap[kb >> 5];
  return prefix[kb >> 5] + __popc(w & ((1u << (kb & 31)) - 1u));
}

// Marks every key block that rows [r0, r1) reference. Entries outside [0, n_cols) are ignored.
__device__ void mark_rows(const int32_t* indptr, const int32_t* indices, int r0, int r1, int n_cols,
                          uint32_t* bitmap) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = r0 + warp; r < r1; r += kWarps) {
    const int e1 = indptr[r + 1];
    for (int e = indptr[r] + lane; e < e1; e += 32) {
      const int c = indices[e];
      if (c >= 0 && c < n_cols) mark(bitmap, c >> 5);
    }
  }
}

__global__ void __launch_bounds__(kThreads) tiles_count_kernel(const int32_t* __restrict__ indptr,
                                                                const int32_t* __restrict__ indices,
                                                                int n_rows, int n_cols, int block_q,
                                                                int32_t* __restrict__ counts) {
  extern __shared__ uint32_t smem[];
  const int words = ((n_cols + 31) / 32 + 31) / 32;
  uint32_t* bitmap = smem;
  for (int i = threadIdx.x; i < words; i += kThreads) bitmap[i] = 0;
  __syncthreads();
  const int qb = blockIdx.x;
  const int r0 = qb * block_q, r1 = min(r0 + block_q, n_rows);
  mark_rows(indptr, indices, r0, r1, n_cols, bitmap);
  __syncthreads();
  int local = 0;
  for (int i = threadIdx.x; i < words; i += kThreads) local += __popc(bitmap[i]);
  __shared__ int part[kWarps];
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) local += __shfl_down_sync(0xffffffffu, local, d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kWarps; ++w) s += part[w];
    counts[qb] = s;
  }
}

// ptr[0] = 0, ptr[i + 1] = ptr[i] + counts[i] (one CTA).
__global__ void __launch_bounds__(1024) exclusive_scan_kernel(const int32_t* __restrict__ counts, int n,
                                                               int32_t* __restrict__ ptr) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
    carry = 0;
    ptr[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < n; base += 1024) {
    const int i = base + tid;
    const int x = i < n ? counts[i] : 0;
    int incl = x;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int s = warp_sums[lane];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, s, d);
        if (lane >= d) s += y;
      }
      warp_sums[lane] = s;
    }
    __syncthreads();
    const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + carry;
    if (i < n) ptr[i + 1] = before + incl;
    __syncthreads();
    if (tid == 1023) carry = before + incl;
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kThreads) tiles_fill_kernel(const int32_t* __restrict__ indptr,
                                                               const int32_t* __restrict__ indices,
                                                               int n_rows, int n_cols, int block_q,
                                                               const int32_t* __restrict__ ptr,
                                                               int32_t* __restrict__ tile_kb,
                                                               uint32_t* __restrict__ tile_bits,
                                                               int word_cap) {
  extern __shared__ uint32_t smem[];
  const int words = ((n_cols + 31) / 32 + 31) / 32;
  uint32_t* bitmap = smem;
  int* prefix = reinterpret_cast<int*>(smem + words);
  uint32_t* acc = smem + 2 * words;  // [word_cap] tile words
  __shared__ int scratch[kWarps];
  for (int i = threadIdx.x; i < words; i += kThreads) bitmap[i] = 0;
  __syncthreads();
  const int qb = blockIdx.x;
  const int r0 = qb * block_q, r1 = min(r0 + block_q, n_rows);
  mark_rows(indptr, indices, r0, r1, n_cols, bitmap);
  __syncthreads();
  bitmap_prefix(bitmap, prefix, words, scratch);
  const int base = ptr[qb];
  const int count = ptr[qb + 1] - base;
  // Key blocks, ascending.
  for (int i = threadIdx.x; i < words; i += kThreads) {
    uint32_t w = bitmap[i];
    int k = prefix[i];
    while (w) {
      const int b = __ffs(w) - 1;
      w &= w - 1;
      if (k < count) tile_kb[base + k] = i * 32 + b;
      ++k;
    }
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwords = count * block_q;
  const bool in_smem = nwords <= word_cap;
  uint32_t* out = tile_bits + static_cast<size_t>(base) * block_q;
  uint32_t* dst = in_smem ? acc : out;
  for (int i = threadIdx.x; i < nwords; i += kThreads) dst[i] = 0;
  __syncthreads();
  for (int r = r0 + warp; r < r1; r += kWarps) {
    const int e1 = indptr[r + 1];
    const int row = r - r0;
    for (int e = indptr[r] + lane; e < e1; e += 32) {
      const int c = indices[e];
      if (c < 0 || c >= n_cols) continue;
      const int t = rank_of(bitmap, prefix, c >> 5);
      if (t < count) atomicOr(&dst[t * block_q + row], 1u << (c & 31));
    }
  }
  __syncthreads();
  if (in_smem) {
    for (int i = threadIdx.x; i < nwords; i += kThreads) out[i] = acc[i];
  }
}

// Paired list, pass 1: number of distinct key blocks of 64-row blocks 2p and 2p+1.
__global__ void __launch_bounds__(kThreads) pair_count_kernel(const int32_t* __restrict__ ptr,
                                                               const int32_t* __restrict__ kb, int n_blocks,
                                                               int n_cols, int32_t* __restrict__ counts) {
  extern __shared__ uint32_t smem[];
  const int words = ((n_cols + 31) / 32 + 31) / 32;
  const int nkb = (n_cols + 31) / 32;
  uint32_t* bitmap = smem;
  for (int i = threadIdx.x; i < words; i += kThreads) bitmap[i] = 0;
  __syncthreads();
  const int p = blockIdx.x;
  const int t0 = ptr[2 * p], t1 = ptr[min(2 * p + 2, n_blocks)];
  for (int t = t0 + threadIdx.x; t < t1; t += kThreads) {
    const int k = kb[t];
    if (k >= 0 && k < nkb) mark(bitmap, k);
  }
  __syncthreads();
  int local = 0;
  for (int i = threadIdx.x; i < words; i += kThreads) local += __popc(bitmap[i]);
  __shared__ int part[kWarps];
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) local += __shfl_down_sync(0xffffffffu, local, d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = local;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kWarps; ++w) s += part[w];
    counts[p] = s;
  }
}

__global__ void __launch_bounds__(kThreads) pair_fill_kernel(const int32_t* __restrict__ ptr,
                                                              const int32_t* __restrict__ kb,
                                                              const uint32_t* __restrict__ bits, int n_blocks,
                                                              int n_cols, const int32_t* __restrict__ ptr2,
                                                              int32_t* __restrict__ kb2,
                                                              uint32_t* __restrict__ bits2) {
  extern __shared__ uint32_t smem[];
  const int words = ((n_cols + 31) / 32 + 31) / 32;
  const int nkb = (n_cols + 31) / 32;
  uint32_t* bitmap = smem;
  int* prefix = reinterpret_cast<int*>(smem + words);
  __shared__ int scratch[kWarps];
  for (int i = threadIdx.x; i < words; i += kThreads) bitmap[i] = 0;
  __syncthreads();
  const int p = blockIdx.x;
  const int t0 = ptr[2 * p], t1 = ptr[min(2 * p + 2, n_blocks)];
  const int tmid = ptr[min(2 * p + 1, n_blocks)];
  for (int t = t0 + threadIdx.x; t < t1; t += kThreads) {
    const int k = kb[t];
    if (k >= 0 && k < nkb) mark(bitmap, k);
  }
  __syncthreads();
  bitmap_prefix(bitmap, prefix, words, scratch);
  const int base = ptr2[p];
  const int count = ptr2[p + 1] - base;
  for (int i = threadIdx.x; i < words; i += kThreads) {
    uint32_t w = bitmap[i];
    int k = prefix[i];
    while (w) {
      const int b = __ffs(w) - 1;
      w &= w - 1;
      if (k < count) kb2[base + k] = i * 32 + b;
      ++k;
    }
  }
  uint32_t* out = bits2 + static_cast<size_t>(base) * 128;
  for (int i = threadIdx.x; i < count * 128; i += kThreads) out[i] = 0;
  __syncthreads();
  // One warp per source tile: 64 words -> rows [half*64, half*64 + 64) of the paired tile.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t = t0 + warp; t < t1; t += kWarps) {
    const int k = kb[t];
    if (k < 0 || k >= nkb) continue;
    const int r = rank_of(bitmap, prefix, k);
    if (r >= count) continue;
    const int half = t >= tmid ? 64 : 0;
    const uint32_t* src = bits + static_cast<size_t>(t) * 64;
    out[r * 128 + half + lane] = src[lane];
    out[r * 128 + half + 32 + lane] = src[32 + lane];
  }
}

// Column mask of a 128-row tile: OR of its 128 words (which of the tile's 32 columns any row uses).
__device__ __forceinline__ uint32_t tile_colmask(const uint32_t* __restrict__ bits2, int e, int lane) {
  const uint4 w = reinterpret_cast<const uint4*>(bits2 + static_cast<size_t>(e) * 128)[lane];
  uint32_t m = w.x | w.y | w.z | w.w;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) m |= __shfl_xor_sync(0xffffffffu, m, d);
  return m;
}

// Gathered list, pass 1: per 128-row block, ceil(distinct used columns / 32) tiles.
__global__ void __launch_bounds__(kThreads) gather_count_kernel(const int32_t* __restrict__ ptr2,
                                                                 const uint32_t* __restrict__ bits2,
                                                                 int32_t* __restrict__ counts) {
  const int p = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = ptr2[p], e1 = ptr2[p + 1];
  int used = 0;
  for (int e = e0 + warp; e < e1; e += kWarps) used += __popc(tile_colmask(bits2, e, lane));
  __shared__ int part[kWarps];
  if (lane == 0) part[warp] = used;
  __syncthreads();
  if (threadIdx.x == 0) {
    int s = 0;
    for (int w = 0; w < kWarps; ++w) s += part[w];
    counts[p] = (s + 31) / 32;
  }
}

// Gathered list, pass 2. Shared memory: colmask[n_sub], base[n_sub], then (if they fit) the block's
// words. A block with more tiles than `max_sub` falls back to recomputing column masks on the fly.
__global__ void __launch_bounds__(kThreads) gather_fill_kernel(const int32_t* __restrict__ ptr2,
                                                                const int32_t* __restrict__ kb2,
                                                                const uint32_t* __restrict__ bits2,
                                                                const int32_t* __restrict__ ptr_g,
                                                                int32_t* __restrict__ cols_g,
                                                                uint32_t* __restrict__ bits_g, int max_sub,
                                                                int word_cap) {
  extern __shared__ uint32_t smem[];
  uint32_t* cm = smem;                                   // [max_sub]
  int* base = reinterpret_cast<int*>(smem + max_sub);    // [max_sub]
  uint32_t* acc = smem + 2 * max_sub;                    // [word_cap]
  __shared__ int scratch[kWarps];
  const int p = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e0 = ptr2[p], n_sub = ptr2[p + 1] - e0;
  const int g0 = ptr_g[p], ng = ptr_g[p + 1] - g0;
  if (n_sub == 0) return;
  if (n_sub > max_sub) return;  // the host sizes max_sub from the largest block, so this never happens
  for (int e = warp; e < n_sub; e += kWarps) {
    const uint32_t m = tile_colmask(bits2, e0 + e, lane);
    if (lane == 0) cm[e] = m;
  }
  __syncthreads();
  // Exclusive scan of popcount(cm) over the block's tiles (reuses the bitmap prefix helper).
  bitmap_prefix(cm, base, n_sub, scratch);
  // Columns: slot base[e] + rank of bit j in cm[e]; padding slots repeat the block's last column.
  int last = 0;
  {
    const int e = n_sub - 1;
    last = kb2[e0 + e] * 32 + (31 - __clz(cm[e] ? cm[e] : 1u));
  }
  int32_t* cols = cols_g + static_cast<size_t>(g0) * 32;
  for (int i = threadIdx.x; i < ng * 32; i += kThreads) cols[i] = last;
  __syncthreads();
  for (int e = warp; e < n_sub; e += kWarps) {
    const uint32_t m = cm[e];
    if ((m >> lane) & 1u) cols[base[e] + __popc(m & ((1u << lane) - 1u))] = kb2[e0 + e] * 32 + lane;
  }
  // Words: OR each (tile, row) word's bits into the slots of its columns.
  const bool in_smem = ng * 128 <= word_cap;
  uint32_t* out = bits_g + static_cast<size_t>(g0) * 128;
  uint32_t* dst = in_smem ? acc : out;
  for (int i = threadIdx.x; i < ng * 128; i += kThreads) dst[i] = 0;
  __syncthreads();
  for (int idx = threadIdx.x; idx < n_sub * 128; idx += kThreads) {
    const int e = idx >> 7, r = idx & 127;
    uint32_t w = bits2[static_cast<size_t>(e0 + e) * 128 + r];
    const uint32_t m = cm[e];
    const int b0 = base[e];
    while (w) {
      const int j = __ffs(w) - 1;
      w &= w - 1;
      const int slot = b0 + __popc(m & ((1u << j) - 1u));
      atomicOr(&dst[(slot >> 5) * 128 + r], 1u << (slot & 31));
    }
  }
  __syncthreads();
  if (in_smem)
    for (int i = threadIdx.x; i < ng * 128; i += kThreads) out[i] = acc[i];
}

// Hilbert-curve index of unit-sphere points (Skilling, "Programming the Hilbert curve", 2004: axes ->
// transpose by undoing excess work per bit plane, Gray encoding, then bit interleaving), the device
// counterpart of hilbert_order's key (pallas_attn.py:41-82). Non-finite points get INT64_MAX.
__global__ void hilbert_codes_kernel(const double* __restrict__ lat_deg, const double* __restrict__ lon_deg, int n,
                                     int bits, long long* __restrict__ codes) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const double kDeg = 3.14159265358979323846 / 180.0;
  const double la = lat_deg[i] * kDeg, lo = lon_deg[i] * kDeg;
  const double xyz[3] = {cos(la) * cos(lo), cos(la) * sin(lo), sin(la)};
  bool finite = true;
  long long x[3];
  const double top = static_cast<double>((1 << bits) - 1);
  for (int a = 0; a < 3; ++a) {
    double v = xyz[a];
    if (!isfinite(v)) {
      finite = false;
      v = 0.0;
    }
    double s = rint((v + 1.0) / 2.0 * top);  // round half to even, as NumPy's round
    s = fmin(fmax(s, 0.0), top);
    x[a] = static_cast<long long>(s);
  }
  if (!finite) {
    codes[i] = 0x7fffffffffffffffll;
    return;
  }
  const long long msb = 1ll << (bits - 1);
  for (long long q = msb; q > 1; q >>= 1) {
    const long long low = q - 1;
    for (int a = 0; a < 3; ++a) {
      if (x[a] & q) {
        x[0] ^= low;
      } else {
        const long long t = (x[0] ^ x[a]) & low;
        x[0] ^= t;
        x[a] ^= t;
      }
    }
  }
  x[1] ^= x[0];
  x[2] ^= x[1];
  long long t = 0;
  for (long long q = msb; q > 1; q >>= 1)
    if (x[2] & q) t ^= q - 1;
  for (int a = 0; a < 3; ++a) x[a] ^= t;
  long long code = 0;
  for (int b = bits - 1; b >= 0; --b)
    for (int a = 0; a < 3; ++a) code = (code << 1) | ((x[a] >> b) & 1);
  codes[i] = code;
}

}  // namespace

cudaError_t launch_hilbert_codes(const double* lat_deg, const double* lon_deg, int n, int bits, long long* codes,
                                 cudaStream_t stream) {
  if (n > 0) hilbert_codes_kernel<<<(n + 255) / 256, 256, 0, stream>>>(lat_deg, lon_deg, n, bits, codes);
  return cudaGetLastError();
}

int tiles_bitmap_words(int n_cols) { return ((n_cols + 31) / 32 + 31) / 32; }

cudaError_t launch_exclusive_scan(const int32_t* counts, int n, int32_t* ptr, cudaStream_t stream) {
  exclusive_scan_kernel<<<1, 1024, 0, stream>>>(counts, n, ptr);
  return cudaGetLastError();
}

cudaError_t launch_gather_count(const int32_t* ptr2, const uint32_t* bits2, int n_blocks, int32_t* ptr_g,
                                int32_t* counts, cudaStream_t stream) {
  if (n_blocks > 0) gather_count_kernel<<<n_blocks, kThreads, 0, stream>>>(ptr2, bits2, counts);
  exclusive_scan_kernel<<<1, 1024, 0, stream>>>(counts, n_blocks, ptr_g);
  return cudaGetLastError();
}

cudaError_t launch_gather_fill(const int32_t* ptr2, const int32_t* kb2, const uint32_t* bits2, int n_blocks,
                               int max_sub, const int32_t* ptr_g, int32_t* cols_g, uint32_t* bits_g,
                               cudaStream_t stream) {
  if (n_blocks == 0) return cudaSuccess;
  max_sub = max_sub < 1 ? 1 : max_sub;
  const size_t fixed = static_cast<size_t>(2 * max_sub) * 4;
  if (fixed > 160 * 1024) return cudaErrorInvalidValue;
  int cap = static_cast<int>((200 * 1024 - fixed) / 4);
  const size_t smem = fixed + static_cast<size_t>(cap) * 4;
  cudaError_t e = cudaFuncSetAttribute(gather_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  gather_fill_kernel<<<n_blocks, kThreads, smem, stream>>>(ptr2, kb2, bits2, ptr_g, cols_g, bits_g, max_sub, cap);
  return cudaGetLastError();
}

cudaError_t launch_tiles_count(const int32_t* indptr, const int32_t* indices, int n_rows, int n_cols,
                               int block_q, int32_t* tile_ptr, int32_t* counts, cudaStream_t stream) {
  const int nqb = (n_rows + block_q - 1) / block_q;
  const size_t smem = static_cast<size_t>(tiles_bitmap_words(n_cols)) * 4;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(tiles_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  if (nqb > 0) tiles_count_kernel<<<nqb, kThreads, smem, stream>>>(indptr, indices, n_rows, n_cols, block_q, counts);
  exclusive_scan_kernel<<<1, 1024, 0, stream>>>(counts, nqb, tile_ptr);
  return cudaGetLastError();
}

cudaError_t launch_tiles_fill(const int32_t* indptr, const int32_t* indices, int n_rows, int n_cols, int block_q,
                              const int32_t* tile_ptr, int32_t* tile_kb, uint32_t* tile_bits,
                              cudaStream_t stream) {
  const int nqb = (n_rows + block_q - 1) / block_q;
  if (nqb == 0) return cudaSuccess;
  const int words = tiles_bitmap_words(n_cols);
  // Shared-memory tile words: up to 96 KB, or what is left under the 200 KB budget.
  int cap = 24 * 1024;
  const size_t fixed = static_cast<size_t>(2 * words) * 4;
  if (fixed + static_cast<size_t>(cap) * 4 > 200 * 1024) cap = static_cast<int>((200 * 1024 - fixed) / 4);
  if (cap < 0) cap = 0;
  const size_t smem = fixed + static_cast<size_t>(cap) * 4;
  cudaError_t e = cudaFuncSetAttribute(tiles_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  tiles_fill_kernel<<<nqb, kThreads, smem, stream>>>(indptr, indices, n_rows, n_cols, block_q, tile_ptr, tile_kb,
                                                      tile_bits, cap);
  return cudaGetLastError();
}

cudaError_t launch_pair_count(const int32_t* ptr, const int32_t* kb, int n_blocks, int n_cols, int32_t* ptr2,
                              int32_t* counts, cudaStream_t stream) {
  const int npb = (n_blocks + 1) / 2;
  const size_t smem = static_cast<size_t>(tiles_bitmap_words(n_cols)) * 4;
  cudaError_t e = cudaFuncSetAttribute(pair_count_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem < 1024 ? 1024 : smem));
  if (e != cudaSuccess) return e;
  if (npb > 0) pair_count_kernel<<<npb, kThreads, smem, stream>>>(ptr, kb, n_blocks, n_cols, counts);
  exclusive_scan_kernel<<<1, 1024, 0, stream>>>(counts, npb, ptr2);
  return cudaGetLastError();
}

cudaError_t launch_pair_fill(const int32_t* ptr, const int32_t* kb, const uint32_t* bits, int n_blocks, int n_cols,
                             const int32_t* ptr2, int32_t* kb2, uint32_t* bits2, cudaStream_t stream) {
  const int npb = (n_blocks + 1) / 2;
  if (npb == 0) return cudaSuccess;
  const size_t smem = static_cast<size_t>(2 * tiles_bitmap_words(n_cols)) * 4;
  cudaError_t e = cudaFuncSetAttribute(pair_fill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem < 1024 ? 1024 : smem));
  if (e != cudaSuccess) return e;
  pair_fill_kernel<<<npb, kThreads, smem, stream>>>(ptr, kb, bits, n_blocks, n_cols, ptr2, kb2, bits2);
  return cudaGetLastError();
}

}  // namespace fwn
