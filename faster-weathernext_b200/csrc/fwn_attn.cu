// C ABI of libfwn_attn.so (include/fwn_attn.h): argument checks, TMA descriptors, kernel launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/fwn_attn.h"
#include "common.cuh"

#include "attn_bwd.cuh"
#include "attn_fwd.cuh"
#include "attn_fwd_wide.cuh"
#include "attn_bwd_wide.cuh"
#include "gemm.cuh"
#include "tiles.cuh"

namespace {

thread_local std::string g_last_error;

fwn_status fail(fwn_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

fwn_status ok() {
  g_last_error.clear();
  return FWN_OK;
}

fwn_status cuda_fail(cudaError_t e, const char* what) {
  return fail(FWN_ERR_LAUNCH, "%s: %s", what, cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  // The driver call needs a current context. A thread whose runtime calls so far needed none (autograd's device
  // thread running a backward whose allocations all came from the caching allocator, for one) has its device set but
  // no context bound: cudaSetDevice on the thread's current device binds that device's primary context (and changes
  // nothing when it is bound already).
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaSetDevice(dev);
  return fn;
}

// 4D map over a [B, n, H, D] tensor (D contiguous): box = 128 bytes of D x 1 head x `rows` nodes x 1.
// `atom32` selects the 128-byte swizzle with 32-byte atoms (tf32 operands read MN-major by the MMA).
fwn_status make_map(CUtensorMap* map, const void* base, const fwn_attn_desc& d, int rows, bool atom32 = false,
                    bool out = false) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FWN_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const int es = d.dtype == FWN_DTYPE_BF16 ? 2 : 4;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d.head_dim), static_cast<cuuint64_t>(d.heads),
                        static_cast<cuuint64_t>(d.n), static_cast<cuuint64_t>(d.batch)};
  const int64_t sh = out ? d.out_stride_h : d.stride_h, sn = out ? d.out_stride_n : d.stride_n,
                sb = out ? d.out_stride_b : d.stride_b;
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(sh) * es, static_cast<cuuint64_t>(sn) * es,
                           static_cast<cuuint64_t>(sb) * es};
  cuuint32_t box[4] = {static_cast<cuuint32_t>(128 / es), 1, static_cast<cuuint32_t>(rows), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, d.dtype == FWN_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                   4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FWN_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return FWN_OK;
}

// Row layout of the 2D view used by gathered loads: 0 node-major, 1 head-major, -1 not expressible.
int gather_layout(const fwn_attn_desc& d, bool out) {
  const int64_t sh = out ? d.out_stride_h : d.stride_h, sn = out ? d.out_stride_n : d.stride_n,
                sb = out ? d.out_stride_b : d.stride_b;
  if ((d.heads == 1 || sn == static_cast<int64_t>(d.heads) * sh) && (d.batch == 1 || sb == static_cast<int64_t>(d.n) * sn))
    return 0;
  if ((d.n == 1 || sh == static_cast<int64_t>(d.n) * sn) && (d.batch == 1 || sb == static_cast<int64_t>(d.heads) * sh))
    return 1;
  return -1;
}

// 2D map over the (batch, node, head) rows of a tensor for tile::gather4: box = 128 bytes x 1 row.
fwn_status make_map_rows(CUtensorMap* map, const void* base, const fwn_attn_desc& d, int layout, bool atom32,
                         bool out) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FWN_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  const int es = d.dtype == FWN_DTYPE_BF16 ? 2 : 4;
  const int64_t row_stride = layout == 0 ? (out ? d.out_stride_h : d.stride_h) : (out ? d.out_stride_n : d.stride_n);
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(d.head_dim),
                        static_cast<cuuint64_t>(d.batch) * static_cast<cuuint64_t>(d.n) * static_cast<cuuint64_t>(d.heads)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride) * es};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / es), 1};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, d.dtype == FWN_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                   2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FWN_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled (rows) failed (%d)", static_cast<int>(r));
  return FWN_OK;
}

fwn_status check_desc(const fwn_attn_desc* d) {
  if (!d) return fail(FWN_ERR_INVALID_ARGUMENT, "desc is null");
  if (d->batch <= 0 || d->heads <= 0 || d->n <= 0)
    return fail(FWN_ERR_INVALID_ARGUMENT, "batch, heads and n must be positive (got %d, %d, %d)", d->batch, d->heads, d->n);
  if (d->head_dim != 64 && d->head_dim != 128)
    return fail(FWN_ERR_UNSUPPORTED, "head_dim %d not built (64 or 128)", d->head_dim);
  if (d->dtype != FWN_DTYPE_BF16 && d->dtype != FWN_DTYPE_F32)
    return fail(FWN_ERR_INVALID_ARGUMENT, "unknown dtype %d", d->dtype);
  if (d->mode == FWN_MODE_BF16 && d->dtype != FWN_DTYPE_BF16)
    return fail(FWN_ERR_INVALID_ARGUMENT, "mode BF16 takes bf16 tensors");
  if ((d->mode == FWN_MODE_TF32 || d->mode == FWN_MODE_TF32X3) && d->dtype != FWN_DTYPE_F32)
    return fail(FWN_ERR_INVALID_ARGUMENT, "modes TF32/TF32X3 take float32 tensors");
  if (d->mode < 0 || d->mode > 2) return fail(FWN_ERR_INVALID_ARGUMENT, "unknown mode %d", d->mode);
  if (!(d->scale > 0.f)) return fail(FWN_ERR_INVALID_ARGUMENT, "scale must be positive");
  const int64_t es = d->dtype == FWN_DTYPE_BF16 ? 2 : 4;
  if ((d->stride_h * es) % 16 || (d->stride_n * es) % 16 || (d->stride_b * es) % 16 ||
      (d->out_stride_h * es) % 16 || (d->out_stride_n * es) % 16 || (d->out_stride_b * es) % 16)
    return fail(FWN_ERR_INVALID_ARGUMENT, "strides must be multiples of 16 bytes");
  if (d->stride_h < d->head_dim || d->stride_n <= 0 || d->stride_b <= 0 || d->out_stride_h < d->head_dim ||
      d->out_stride_n <= 0 || d->out_stride_b <= 0)
    return fail(FWN_ERR_INVALID_ARGUMENT, "strides must be positive and rows must not overlap");
  if (d->flags & ~static_cast<int32_t>(FWN_DESC_GRAD_STRIDES))
    return fail(FWN_ERR_INVALID_ARGUMENT, "unknown desc flags 0x%x", static_cast<unsigned>(d->flags));
  if (d->flags & FWN_DESC_GRAD_STRIDES) {
    if ((d->grad_stride_h * es) % 16 || (d->grad_stride_n * es) % 16 || (d->grad_stride_b * es) % 16)
      return fail(FWN_ERR_INVALID_ARGUMENT, "gradient strides must be multiples of 16 bytes");
    if (d->grad_stride_h < d->head_dim || d->grad_stride_n <= 0 || d->grad_stride_b <= 0)
      return fail(FWN_ERR_INVALID_ARGUMENT, "gradient strides must be positive and rows must not overlap");
  }
  return FWN_OK;
}

// The descriptor with its gradient strides resolved (the out strides unless FWN_DESC_GRAD_STRIDES is set). Reads
// the grad_stride fields only when the flag is set: a caller's struct may end at out_stride_h.
fwn_attn_desc resolve_grad_strides(const fwn_attn_desc* desc) {
  fwn_attn_desc d;
  std::memcpy(&d, desc, offsetof(fwn_attn_desc, grad_stride_b));
  const bool own = (desc->flags & FWN_DESC_GRAD_STRIDES) != 0;
  d.grad_stride_b = own ? desc->grad_stride_b : d.out_stride_b;
  d.grad_stride_n = own ? desc->grad_stride_n : d.out_stride_n;
  d.grad_stride_h = own ? desc->grad_stride_h : d.out_stride_h;
  return d;
}

fwn_status check_tiles(const fwn_tile_list* t, const fwn_attn_desc* d, const char* name) {
  if (!t) return fail(FWN_ERR_INVALID_ARGUMENT, "%s is null", name);
  if (t->block_rows != 128)
    return fail(FWN_ERR_INVALID_ARGUMENT, "%s: attention kernels take the 128-row list (fwn_tiles_pair_*), got %d rows",
                name, t->block_rows);
  if (t->n_blocks != (d->n + 127) / 128)
    return fail(FWN_ERR_INVALID_ARGUMENT, "%s: %d blocks for n=%d (expected %d)", name, t->n_blocks, d->n, (d->n + 127) / 128);
  if (!t->ptr || (t->n_tiles > 0 && ((!t->kb && !t->cols) || !t->bits)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(t->bits)) return fail(FWN_ERR_INVALID_ARGUMENT, "%s: bits must be 16-byte aligned", name);
  if (t->cols && t->n_tiles > 0 && !aligned16(t->cols))
    return fail(FWN_ERR_INVALID_ARGUMENT, "%s: cols must be 16-byte aligned", name);
  if (t->n_cols > d->n) return fail(FWN_ERR_INVALID_ARGUMENT, "%s: %d mask columns > n=%d", name, t->n_cols, d->n);
  return FWN_OK;
}

// SMs of the current device (queried per call: a process may drive several devices).
int num_sms() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return 148;
  return sms;
}

// Resident CTAs per SM from the device limits: shared memory (plus the per-block reservation), registers
// (allocated per warp in units of 256), threads, and tensor memory (512 columns per SM; an allocation that
// cannot be satisfied waits for a resident CTA to free its columns). The runtime occupancy query reports
// one CTA per SM for these kernels where two fit by all of these limits, so it is not used.
template <typename Kernel>
fwn_status persistent_grid(Kernel kernel, int threads, int smem, int tmem_cols, int items, int* grid) {
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(carveout)");
  cudaFuncAttributes fa;
  if ((e = cudaFuncGetAttributes(&fa, kernel)) != cudaSuccess) return cuda_fail(e, "cudaFuncGetAttributes");
  int dev = 0, smem_sm = 0, reserved = 0, regs_sm = 0, threads_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
  cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
  cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
  cudaDeviceGetAttribute(&threads_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
  const int warps = (threads + 31) / 32;
  const int regs_warp = ((fa.numRegs * 32 + 255) / 256) * 256;
  int per_sm = smem_sm / (smem + static_cast<int>(fa.sharedSizeBytes) + reserved);
  per_sm = std::min(per_sm, regs_sm / std::max(1, regs_warp * warps));
  per_sm = std::min(per_sm, threads_sm / threads);
  per_sm = std::min(per_sm, 512 / tmem_cols);
  if (per_sm < 1) return fail(FWN_ERR_LAUNCH, "kernel does not fit on an SM");
  *grid = items < per_sm * num_sms() ? items : per_sm * num_sms();
  return FWN_OK;
}

// Delta rows of fwn_attn_bwd_noalloc: a fixed array in every device that loads this library, so that
// callers without an allocator can run the backward (4 MiB per device, held until the process exits).
// Host code cannot use the symbol as a pointer; its device address is looked up once per device.
static __device__ __align__(256) float g_noalloc_delta[FWN_NOALLOC_DELTA_ROWS];

std::mutex g_noalloc_mutex;
constexpr int kMaxDevices = 64;
float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_delta on the current device (looked up on the first call per device and kept:
// valid while the device's primary context lives, i.e. until a cudaDeviceReset, after which the header forbids
// further calls on that device).
fwn_status noalloc_delta(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(FWN_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (!g_noalloc_ptr[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_noalloc_delta);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(delta scratch)");
    g_noalloc_ptr[dev] = static_cast<float*>(ptr);
  }
  *out = g_noalloc_ptr[dev];
  return FWN_OK;
}

#ifdef FWN_TRACE
unsigned long long* g_trace = nullptr;
unsigned long long* trace_buffer_peek() { return g_trace; }
// Trace builds: one device buffer of kTraceCtas x kTraceEvents records, cleared per launch.
unsigned long long* trace_buffer() {
  if (!g_trace) cudaMalloc(&g_trace, sizeof(unsigned long long) * fwn::kTraceCtas * fwn::kTraceEvents);
  cudaMemset(g_trace, 0, sizeof(unsigned long long) * fwn::kTraceCtas * fwn::kTraceEvents);
  return g_trace;
}
#endif

template <int D, bool F32, bool GATHER, bool X3 = false>
fwn_status launch_fwd(const fwn_attn_desc& d, const void* q, const void* k, const void* v, const fwn_tile_list& t,
                      void* o, float* lse, int layout, cudaStream_t stream,
                      unsigned long long wait_limit_ns = fwn::kWaitLimitNs, int fault_skip_kv = 0) {
  using C = fwn::FwdCfg<D, F32, X3>;
  CUtensorMap tq, tk, tv, tk32, tv32;
  fwn_status s;
  if ((s = make_map(&tq, q, d, C::ROWS)) != FWN_OK) return s;
  // 4D maps of 32-row boxes: the tile loads of the 32-key lists, and in gathered mode the tiles whose keys are
  // consecutive.
  if ((s = make_map(&tk32, k, d, C::SUB)) != FWN_OK) return s;
  if ((s = make_map(&tv32, v, d, C::SUB, F32)) != FWN_OK) return s;
  if (GATHER) {
    if ((s = make_map_rows(&tk, k, d, layout, false, false)) != FWN_OK) return s;
    if ((s = make_map_rows(&tv, v, d, layout, F32, false)) != FWN_OK) return s;
  } else {
    tk = tk32;
    tv = tv32;
  }
  fwn::FwdParams p{};
  p.ptr2 = t.ptr;
  p.kb2 = t.kb;
  p.cols = t.cols;
  p.bits2 = t.bits;
  p.head_major = layout == 1;
  p.o = o;
  p.lse = lse;
  p.o_sb = d.out_stride_b;
  p.o_sn = d.out_stride_n;
  p.o_sh = d.out_stride_h;
  p.batch = d.batch;
  p.heads = d.heads;
  p.n = d.n;
  p.np = t.n_blocks;
  p.lse_rows = fwn_lse_rows(d.n);
  p.n_items = d.batch * d.heads * t.n_blocks;
  p.scale_log2 = d.scale * 1.4426950408889634f;
  p.q = q;
  p.q_sb = d.stride_b;
  p.q_sn = d.stride_n;
  p.q_sh = d.stride_h;
  p.wait_limit_ns = wait_limit_ns;
  p.fault_skip_kv = fault_skip_kv;
#ifdef FWN_TRACE
  p.trace = trace_buffer();
#endif
  auto kernel = fwn::attn_fwd_kernel<D, F32, GATHER, X3>;
  int grid = 0;
  if ((s = persistent_grid(kernel, C::THREADS, C::SMEM_BYTES, C::TMEM_COLS, p.n_items, &grid)) != FWN_OK) return s;
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tq, tk, tv, tk32, tv32, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd launch");
  return ok();
}

// Wide-chunk forward (bf16, 128-row tile lists): 32- and 128-row K / V boxes, one CTA per SM.
template <int D>
fwn_status launch_fwd_wide(const fwn_attn_desc& d, const void* q, const void* k, const void* v,
                           const fwn_tile_list& t, void* o, float* lse, cudaStream_t stream) {
  using C = fwn::WideCfg<D>;
  CUtensorMap tq, tk, tv, tk4, tv4;
  fwn_status s;
  if ((s = make_map(&tq, q, d, C::ROWS)) != FWN_OK) return s;
  if ((s = make_map(&tk, k, d, C::SUB)) != FWN_OK) return s;
  if ((s = make_map(&tv, v, d, C::SUB)) != FWN_OK) return s;
  if ((s = make_map(&tk4, k, d, C::KEYS)) != FWN_OK) return s;
  if ((s = make_map(&tv4, v, d, C::KEYS)) != FWN_OK) return s;
  fwn::FwdParams p{};
  p.ptr2 = t.ptr;
  p.kb2 = t.kb;
  p.bits2 = t.bits;
  p.o = o;
  p.lse = lse;
  p.o_sb = d.out_stride_b;
  p.o_sn = d.out_stride_n;
  p.o_sh = d.out_stride_h;
  p.batch = d.batch;
  p.heads = d.heads;
  p.n = d.n;
  p.np = t.n_blocks;
  p.lse_rows = fwn_lse_rows(d.n);
  p.n_items = d.batch * d.heads * t.n_blocks;
  p.scale_log2 = d.scale * 1.4426950408889634f;
#ifdef FWN_TRACE
  p.trace = trace_buffer();
#endif
  auto kernel = fwn::attn_fwd_wide_kernel<D>;
  int grid = 0;
  if ((s = persistent_grid(kernel, C::THREADS, C::SMEM_BYTES, C::TMEM_COLS, p.n_items, &grid)) != FWN_OK) return s;
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(tq, tk, tv, tk4, tv4, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "attn_fwd_wide launch");
  return ok();
}

// Dense lists (on average at least 16 tiles of 32 keys per 128-row block) and head_dim 128 take the
// wide-chunk forward in bf16 with 32-key tile lists.
bool use_wide(const fwn_attn_desc& d, const fwn_tile_list& t) {
  if (d.mode != FWN_MODE_BF16 || t.cols) return false;
  return d.head_dim == 128 || static_cast<int64_t>(t.n_tiles) >= 16 * static_cast<int64_t>(t.n_blocks);
}

template <int KIND, int D, bool F32, int CH, bool GATHER, bool X3>
fwn_status launch_bwd_pass(const fwn_attn_desc& d, const void* q, const void* k, const void* v, const void* d_o,
                           const float* lse, const float* delta, const fwn_tile_list& t, void* out0, void* out1,
                           int layout, cudaStream_t stream) {
  using C = fwn::BwdCfg<KIND, D, F32, CH, X3>;
  constexpr bool kKeys = KIND != fwn::kBwdDQ;
  CUtensorMap r0, r1, c0, c1, c0mn, c1mn;
  fwn_status s;
  // dQ pass: rows Q, dO; columns K, V.   dK / dV passes: rows K, V; columns Q, dO.
  const void* rp0 = kKeys ? k : q;
  const void* rp1 = kKeys ? v : d_o;
  const void* cp0 = kKeys ? q : k;
  const void* cp1 = kKeys ? d_o : v;
  const bool r1_out = !kKeys, c1_out = kKeys;
  if ((s = make_map(&r0, rp0, d, C::ROWS)) != FWN_OK) return s;
  if ((s = make_map(&r1, rp1, d, C::ROWS, false, r1_out)) != FWN_OK) return s;
  if (GATHER) {
    if ((s = make_map_rows(&c0, cp0, d, layout, false, false)) != FWN_OK) return s;
    if ((s = make_map_rows(&c1, cp1, d, layout, false, c1_out)) != FWN_OK) return s;
  } else {
    if ((s = make_map(&c0, cp0, d, C::SUB)) != FWN_OK) return s;
    if ((s = make_map(&c1, cp1, d, C::SUB, false, c1_out)) != FWN_OK) return s;
  }
  c0mn = c0;
  c1mn = c1;
  if (F32) {
    if (GATHER) {
      if ((s = make_map_rows(&c0mn, cp0, d, layout, true, false)) != FWN_OK) return s;
      if ((s = make_map_rows(&c1mn, cp1, d, layout, true, c1_out)) != FWN_OK) return s;
    } else {
      if ((s = make_map(&c0mn, cp0, d, C::SUB, true)) != FWN_OK) return s;
      if ((s = make_map(&c1mn, cp1, d, C::SUB, true, c1_out)) != FWN_OK) return s;
    }
  }
  // 32-row 4D maps for gathered tiles whose columns are consecutive (the tile-mode maps themselves otherwise).
  CUtensorMap c0r = c0, c1r = c1, c0mnr = c0mn, c1mnr = c1mn;
  if (GATHER) {
    if ((s = make_map(&c0r, cp0, d, C::SUB)) != FWN_OK) return s;
    if ((s = make_map(&c1r, cp1, d, C::SUB, false, c1_out)) != FWN_OK) return s;
    if (F32) {
      if ((s = make_map(&c0mnr, cp0, d, C::SUB, true)) != FWN_OK) return s;
      if ((s = make_map(&c1mnr, cp1, d, C::SUB, true, c1_out)) != FWN_OK) return s;
    } else {
      c0mnr = c0r;
      c1mnr = c1r;
    }
  }
  fwn::BwdParams p{};
  p.ptr2 = t.ptr;
  p.kb2 = t.kb;
  p.cols = t.cols;
  p.bits2 = t.bits;
  p.head_major = layout == 1;
  p.lse = lse;
  p.delta = delta;
  p.out0 = out0;
  p.out1 = out1;
  p.o_sb = d.grad_stride_b;  // dq / dk / dv stores
  p.o_sn = d.grad_stride_n;
  p.o_sh = d.grad_stride_h;
  p.heads = d.heads;
  p.n = d.n;
  p.np = t.n_blocks;
  p.lse_rows = fwn_lse_rows(d.n);
  p.n_items = d.batch * d.heads * t.n_blocks;
  p.scale = d.scale;
  p.scale_log2 = d.scale * 1.4426950408889634f;
  p.r0 = rp0;
  p.r1 = rp1;
  p.r0_sb = d.stride_b;
  p.r0_sn = d.stride_n;
  p.r0_sh = d.stride_h;
  p.r1_sb = r1_out ? d.out_stride_b : d.stride_b;
  p.r1_sn = r1_out ? d.out_stride_n : d.stride_n;
  p.r1_sh = r1_out ? d.out_stride_h : d.stride_h;
#ifdef FWN_TRACE
  p.trace = trace_buffer();
#endif
  auto kernel = fwn::attn_bwd_kernel<KIND, D, F32, CH, GATHER, X3>;
  int grid = 0;
  if ((s = persistent_grid(kernel, C::THREADS, C::SMEM_BYTES, C::TMEM_COLS, p.n_items, &grid)) != FWN_OK) return s;
  // Programmatic serialization: the launch and prologue may overlap the end of the kernel before it in the stream
  // (the delta pass); the kernel waits for that kernel (griddepcontrol.wait) before its first dependent read.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(C::THREADS);
  cfg.dynamicSmemBytes = C::SMEM_BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, r0, r1, c0, c1, c0mn, c1mn, c0r, c1r, c0mnr, c1mnr, p);
  if (e == cudaSuccess) e = cudaGetLastError();
  static const char* const kNames[] = {"attn_bwd dq launch", "attn_bwd dkv launch", "attn_bwd dv launch",
                                       "attn_bwd dk launch"};
  if (e != cudaSuccess) return cuda_fail(e, kNames[KIND]);
  return FWN_OK;
}

// Wide-chunk backward pass (bf16, 128-row tile lists): rows 128-row boxes, columns 32- and 128-row boxes.
template <int KIND, int D>
fwn_status launch_bwd_wide(const fwn_attn_desc& d, const void* q, const void* k, const void* v, const void* d_o,
                           const float* lse, const float* delta, const fwn_tile_list& t, void* out0, void* out1,
                           cudaStream_t stream) {
  using C = fwn::BwdWideCfg<KIND, D>;
  constexpr bool kKeys = KIND != fwn::kBwdDQ;
  CUtensorMap r0, r1, c0, c1, c0w, c1w;
  fwn_status s;
  const void* rp0 = kKeys ? k : q;
  const void* rp1 = kKeys ? v : d_o;
  const void* cp0 = kKeys ? q : k;
  const void* cp1 = kKeys ? d_o : v;
  const bool r1_out = !kKeys, c1_out = kKeys;
  if ((s = make_map(&r0, rp0, d, C::ROWS)) != FWN_OK) return s;
  if ((s = make_map(&r1, rp1, d, C::ROWS, false, r1_out)) != FWN_OK) return s;
  if ((s = make_map(&c0, cp0, d, C::SUB)) != FWN_OK) return s;
  if ((s = make_map(&c1, cp1, d, C::SUB, false, c1_out)) != FWN_OK) return s;
  if ((s = make_map(&c0w, cp0, d, C::COLS)) != FWN_OK) return s;
  if ((s = make_map(&c1w, cp1, d, C::COLS, false, c1_out)) != FWN_OK) return s;
  fwn::BwdParams p{};
  p.ptr2 = t.ptr;
  p.kb2 = t.kb;
  p.bits2 = t.bits;
  p.lse = lse;
  p.delta = delta;
  p.out0 = out0;
  p.out1 = out1;
  p.o_sb = d.grad_stride_b;  // dq / dk / dv stores
  p.o_sn = d.grad_stride_n;
  p.o_sh = d.grad_stride_h;
  p.heads = d.heads;
  p.n = d.n;
  p.np = t.n_blocks;
  p.lse_rows = fwn_lse_rows(d.n);
  p.n_items = d.batch * d.heads * t.n_blocks;
  p.scale = d.scale;
  p.scale_log2 = d.scale * 1.4426950408889634f;
#ifdef FWN_TRACE
  p.trace = trace_buffer();
#endif
  auto kernel = fwn::attn_bwd_wide_kernel<KIND, D>;
  int grid = 0;
  if ((s = persistent_grid(kernel, C::THREADS, C::SMEM_BYTES, C::TMEM_COLS, p.n_items, &grid)) != FWN_OK) return s;
  kernel<<<grid, C::THREADS, C::SMEM_BYTES, stream>>>(r0, r1, c0, c1, c0w, c1w, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, KIND == fwn::kBwdDQ ? "attn_bwd_wide dq launch" : "attn_bwd_wide dkv launch");
  return FWN_OK;
}

// Gathered-mode layout for the column operands of one pass (-1: not gatherable).
int pass_layout(const fwn_attn_desc& d, bool keys) {
  const int a = gather_layout(d, false);
  if (!keys) return a;                   // columns K, V (input strides)
  const int b = gather_layout(d, true);  // columns Q (input) and dO (output strides)
  return (a >= 0 && a == b) ? a : -1;
}

template <int KIND, int D, bool F32, int CH, bool X3 = false>
fwn_status launch_bwd_pass_any(const fwn_attn_desc& d, const void* q, const void* k, const void* v, const void* d_o,
                               const float* lse, const float* delta, const fwn_tile_list& t, void* out0, void* out1,
                               cudaStream_t stream) {
  if (t.cols) {
    const int layout = pass_layout(d, KIND != fwn::kBwdDQ);
    if (layout < 0) return fail(FWN_ERR_INVALID_ARGUMENT, "gathered lists need a node-major or head-major packed layout");
    return launch_bwd_pass<KIND, D, F32, CH, true, X3>(d, q, k, v, d_o, lse, delta, t, out0, out1, layout, stream);
  }
  return launch_bwd_pass<KIND, D, F32, CH, false, X3>(d, q, k, v, d_o, lse, delta, t, out0, out1, 0, stream);
}

template <int D, bool F32>
fwn_status launch_delta(const fwn_attn_desc& d, const void* o, const void* d_o, float* delta, cudaStream_t stream) {
  const int lse_rows = fwn_lse_rows(d.n);
  const int total = d.batch * d.heads * lse_rows;
  constexpr int rows_per_warp = 32 / (D * (F32 ? 4 : 2) / 16);
  const int warps = (total + rows_per_warp - 1) / rows_per_warp;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((warps * 32 + 255) / 256));
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap the launch with the forward's tail
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, fwn::delta_kernel<F32, D>, o, d_o, delta, static_cast<int>(d.heads),
                                     static_cast<int>(d.n), lse_rows, static_cast<int64_t>(d.out_stride_b),
                                     static_cast<int64_t>(d.out_stride_n), static_cast<int64_t>(d.out_stride_h), total);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "delta launch");
  return FWN_OK;
}

// Which backward launches to issue.
enum BwdParts { kDelta = 1, kDq = 2, kDkv = 4, kAll = 7 };

template <int D, bool F32, bool X3 = false>
fwn_status launch_bwd(const fwn_attn_desc& d, const void* q, const void* k, const void* v, const void* o,
                      const float* lse, const void* d_o, const fwn_tile_list* t, const fwn_tile_list* tt, void* dq,
                      void* dk, void* dv, float* delta, int parts, cudaStream_t stream) {
  // 32-column chunks. (64-column chunks with N = 64 S / dP MMAs were measured for tf32 at head_dim 64, where one
  // CTA per SM has the TMEM columns: dQ 3 % faster, dK/dV 8 % slower with half the column stages.)
  constexpr int CH = 1;
  // dV and dK as separate passes where one dK/dV pass does not fit: 3xTF32 and tf32 at head_dim 128 (shared
  // memory), bf16 at head_dim 128 (dK and dV accumulators plus S and dP exceed the 256 TMEM columns of a CTA
  // that shares its SM).
  constexpr bool kSplit = X3 || D == 128;
  fwn_status s;
  if ((parts & kDelta) && (s = launch_delta<D, F32>(d, o, d_o, delta, stream)) != FWN_OK) return s;
  if constexpr (!F32) {
    // Dense lists and head_dim 128 (32-key tile lists): the wide-chunk passes.
    if ((parts & kDq) && use_wide(d, *t)) {
      if ((s = launch_bwd_wide<fwn::kBwdDQ, D>(d, q, k, v, d_o, lse, delta, *t, dq, nullptr, stream)) != FWN_OK) return s;
      parts &= ~kDq;
    }
    if ((parts & kDkv) && use_wide(d, *tt)) {
      // dK and dV in one pass (P / dS written over S / dP in TMEM).
      if ((s = launch_bwd_wide<fwn::kBwdDKV, D>(d, q, k, v, d_o, lse, delta, *tt, dk, dv, stream)) != FWN_OK) return s;
      parts &= ~kDkv;
    }
  }
  if ((parts & kDq) &&
      (s = launch_bwd_pass_any<fwn::kBwdDQ, D, F32, CH, X3>(d, q, k, v, d_o, lse, delta, *t, dq, nullptr, stream)) != FWN_OK)
    return s;
  if (parts & kDkv) {
    if constexpr (kSplit) {
      if ((s = launch_bwd_pass_any<fwn::kBwdDV, D, F32, CH, X3>(d, q, k, v, d_o, lse, delta, *tt, nullptr, dv, stream)) !=
          FWN_OK)
        return s;
      if ((s = launch_bwd_pass_any<fwn::kBwdDK, D, F32, CH, X3>(d, q, k, v, d_o, lse, delta, *tt, dk, nullptr, stream)) !=
          FWN_OK)
        return s;
    } else if ((s = launch_bwd_pass_any<fwn::kBwdDKV, D, F32, CH>(d, q, k, v, d_o, lse, delta, *tt, dk, dv, stream)) !=
               FWN_OK) {
      return s;
    }
  }
  return ok();
}

fwn_status bwd_dispatch(const fwn_attn_desc* desc, const void* q, const void* k, const void* v, const void* o,
                        const float* lse, const void* d_o, const fwn_tile_list* tiles, const fwn_tile_list* tiles_t,
                        void* dq, void* dk, void* dv, const void* ws, size_t ws_bytes, int parts, void* stream);

}  // namespace

extern "C" {

const char* fwn_version(void) { return "fwn_attn 0.1.0 (sm_100a)"; }

const char* fwn_last_error_string(void) { return g_last_error.c_str(); }

int32_t fwn_lse_rows(int32_t n) { return ((n + 127) / 128) * 128; }

fwn_status fwn_device_error(void* stream, int32_t* code) {
  if (!code) return fail(FWN_ERR_INVALID_ARGUMENT, "code is null");
  cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaStreamSynchronize");
  unsigned int word = 0, zero = 0;
  e = cudaMemcpyFromSymbol(&word, fwn::g_device_error, sizeof(word));
  if (e != cudaSuccess) return cuda_fail(e, "read device error word");
  e = cudaMemcpyToSymbol(fwn::g_device_error, &zero, sizeof(zero));
  if (e != cudaSuccess) return cuda_fail(e, "clear device error word");
  *code = !word ? 0 : (word & 0x400u) ? FWN_ERR_INVALID_ARGUMENT : FWN_ERR_DEVICE_TIMEOUT;
  return ok();
}

fwn_status fwn_tiles_workspace_size(int32_t n_rows, int32_t n_cols, int32_t block_q, size_t* bytes) {
  if (!bytes) return fail(FWN_ERR_INVALID_ARGUMENT, "bytes is null");
  if (n_rows < 0 || n_cols < 0 || (block_q != 64 && block_q != 128))
    return fail(FWN_ERR_INVALID_ARGUMENT, "bad shape (n_rows=%d, n_cols=%d, block_q=%d)", n_rows, n_cols, block_q);
  const size_t nqb = (static_cast<size_t>(n_rows) + block_q - 1) / block_q;
  *bytes = ((nqb * 4 + 255) / 256) * 256 + 256;
  return ok();
}

static fwn_status check_csr(const int32_t* indptr, const int32_t* indices, int32_t n_rows, int32_t n_cols,
                            int32_t block_q) {
  if (n_rows < 0 || n_cols < 0) return fail(FWN_ERR_INVALID_ARGUMENT, "negative shape");
  if (block_q != 64 && block_q != 128) return fail(FWN_ERR_INVALID_ARGUMENT, "block_q must be 64 or 128 (got %d)", block_q);
  if (n_cols > (1 << 24)) return fail(FWN_ERR_UNSUPPORTED, "n_cols %d > 2^24", n_cols);
  // indices may be null when the mask has no entries (indptr all zero): it is only read at [indptr[r], indptr[r+1]).
  if (!indptr) return fail(FWN_ERR_INVALID_ARGUMENT, "indptr is null");
  return FWN_OK;
}

fwn_status fwn_tiles_count(const int32_t* indptr, const int32_t* indices, int32_t n_rows, int32_t n_cols,
                           int32_t block_q, int32_t* tile_ptr, void* ws, size_t ws_bytes, void* stream) {
  fwn_status s = check_csr(indptr, indices, n_rows, n_cols, block_q);
  if (s != FWN_OK) return s;
  if (!tile_ptr) return fail(FWN_ERR_INVALID_ARGUMENT, "tile_ptr is null");
  size_t need = 0;
  fwn_tiles_workspace_size(n_rows, n_cols, block_q, &need);
  if (!ws || ws_bytes < need) return fail(FWN_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaError_t e = fwn::launch_tiles_count(indptr, indices, n_rows, n_cols, block_q, tile_ptr,
                                          static_cast<int32_t*>(ws), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tiles_count");
  return ok();
}

fwn_status fwn_tiles_fill(const int32_t* indptr, const int32_t* indices, int32_t n_rows, int32_t n_cols,
                          int32_t block_q, const int32_t* tile_ptr, int32_t* tile_kb, uint32_t* tile_bits,
                          void* stream) {
  fwn_status s = check_csr(indptr, indices, n_rows, n_cols, block_q);
  if (s != FWN_OK) return s;
  if (!tile_ptr || !tile_kb || !tile_bits) return fail(FWN_ERR_INVALID_ARGUMENT, "null output pointer");
  cudaError_t e = fwn::launch_tiles_fill(indptr, indices, n_rows, n_cols, block_q, tile_ptr, tile_kb, tile_bits,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "tiles_fill");
  return ok();
}

fwn_status fwn_tiles_pair_count(const fwn_tile_list* t, int32_t* ptr2, void* ws, size_t ws_bytes, void* stream) {
  if (!t || !ptr2) return fail(FWN_ERR_INVALID_ARGUMENT, "null argument");
  if (t->block_rows != 64) return fail(FWN_ERR_INVALID_ARGUMENT, "pairing takes a 64-row list (got %d)", t->block_rows);
  if (!t->ptr || (t->n_tiles > 0 && !t->kb)) return fail(FWN_ERR_INVALID_ARGUMENT, "null tile pointer");
  if (t->n_cols < 0 || t->n_cols > (1 << 24)) return fail(FWN_ERR_INVALID_ARGUMENT, "bad n_cols %d", t->n_cols);
  const size_t need = ((static_cast<size_t>((t->n_blocks + 1) / 2) * 4 + 255) / 256) * 256 + 256;
  if (!ws || ws_bytes < need) return fail(FWN_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaError_t e = fwn::launch_pair_count(t->ptr, t->kb, t->n_blocks, t->n_cols, ptr2, static_cast<int32_t*>(ws),
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pair_count");
  return ok();
}

fwn_status fwn_tiles_pair_fill(const fwn_tile_list* t, const int32_t* ptr2, int32_t* kb2, uint32_t* bits2,
                               void* stream) {
  if (!t || !ptr2 || !kb2 || !bits2) return fail(FWN_ERR_INVALID_ARGUMENT, "null argument");
  if (t->block_rows != 64) return fail(FWN_ERR_INVALID_ARGUMENT, "pairing takes a 64-row list (got %d)", t->block_rows);
  if (!t->ptr || (t->n_tiles > 0 && (!t->kb || !t->bits))) return fail(FWN_ERR_INVALID_ARGUMENT, "null tile pointer");
  cudaError_t e = fwn::launch_pair_fill(t->ptr, t->kb, t->bits, t->n_blocks, t->n_cols, ptr2, kb2, bits2,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "pair_fill");
  return ok();
}

fwn_status fwn_tiles_gather_count(const fwn_tile_list* t, int32_t* ptr_g, void* ws, size_t ws_bytes, void* stream) {
  if (!t || !ptr_g) return fail(FWN_ERR_INVALID_ARGUMENT, "null argument");
  if (t->block_rows != 128 || t->cols) return fail(FWN_ERR_INVALID_ARGUMENT, "gathering takes a 128-row (paired) list");
  if (!t->ptr || (t->n_tiles > 0 && !t->bits)) return fail(FWN_ERR_INVALID_ARGUMENT, "null tile pointer");
  if (t->n_tiles > 0 && !aligned16(t->bits)) return fail(FWN_ERR_INVALID_ARGUMENT, "bits must be 16-byte aligned");
  const size_t need = ((static_cast<size_t>(t->n_blocks) * 4 + 255) / 256) * 256 + 256;
  if (!ws || ws_bytes < need) return fail(FWN_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaError_t e = fwn::launch_gather_count(t->ptr, t->bits, t->n_blocks, ptr_g, static_cast<int32_t*>(ws),
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather_count");
  return ok();
}

fwn_status fwn_tiles_gather_fill(const fwn_tile_list* t, int32_t max_block_tiles, const int32_t* ptr_g, int32_t* cols_g,
                                 uint32_t* bits_g, void* stream) {
  if (!t || !ptr_g || !cols_g || !bits_g) return fail(FWN_ERR_INVALID_ARGUMENT, "null argument");
  if (t->block_rows != 128 || t->cols) return fail(FWN_ERR_INVALID_ARGUMENT, "gathering takes a 128-row (paired) list");
  if (!t->ptr || (t->n_tiles > 0 && (!t->kb || !t->bits))) return fail(FWN_ERR_INVALID_ARGUMENT, "null tile pointer");
  if (max_block_tiles < 0 || max_block_tiles > 40960)
    return fail(FWN_ERR_INVALID_ARGUMENT, "max_block_tiles %d outside [0, 40960]", max_block_tiles);
  cudaError_t e = fwn::launch_gather_fill(t->ptr, t->kb, t->bits, t->n_blocks, max_block_tiles, ptr_g, cols_g, bits_g,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather_fill");
  return ok();
}

fwn_status fwn_hilbert_codes(const double* lat_deg, const double* lon_deg, int32_t n, int32_t bits, int64_t* codes,
                             void* stream) {
  if (n < 0 || bits < 1 || bits > 20) return fail(FWN_ERR_INVALID_ARGUMENT, "bad n=%d or bits=%d", n, bits);
  if (n > 0 && (!lat_deg || !lon_deg || !codes)) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  cudaError_t e = fwn::launch_hilbert_codes(lat_deg, lon_deg, n, bits, reinterpret_cast<long long*>(codes),
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "hilbert_codes");
  return ok();
}

namespace {

fwn_status cond_layernorm(const float* x, float* x_out, int64_t rows, int32_t d, int32_t rows_per_sample,
                          const int32_t* out_node, const float* scale_offset, float eps, void* out, int32_t out_dtype,
                          void* stream, const void* residual = nullptr) {
  if (rows < 0 || rows_per_sample <= 0 || !(eps > 0.f))
    return fail(FWN_ERR_INVALID_ARGUMENT, "bad rows=%lld, rows_per_sample=%d or eps", static_cast<long long>(rows),
                rows_per_sample);
  if (d != 128 && d != 256 && d != 512 && d != 1024) return fail(FWN_ERR_UNSUPPORTED, "d=%d not built", d);
  if (out_dtype != FWN_DTYPE_BF16 && out_dtype != FWN_DTYPE_F32)
    return fail(FWN_ERR_INVALID_ARGUMENT, "unknown out dtype %d", out_dtype);
  if (rows > 0 && (!x || !scale_offset || !out)) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  if (rows > 0 && (!aligned16(x) || !aligned16(scale_offset) || !aligned16(out)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  if (rows % rows_per_sample != 0)
    return fail(FWN_ERR_INVALID_ARGUMENT, "rows=%lld is not a multiple of rows_per_sample=%d",
                static_cast<long long>(rows), rows_per_sample);
  if (residual && rows > 0 && (!aligned16(residual) || !x_out || !aligned16(x_out)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "residual and x_out must be non-null and 16-byte aligned");
  cudaError_t e = fwn::launch_cond_layernorm(x, x_out, rows, d, rows_per_sample, out_node, scale_offset, eps, out,
                                             out_dtype == FWN_DTYPE_BF16, residual, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cond_layernorm");
  return ok();
}

}  // namespace

fwn_status fwn_cond_layernorm(const float* x, int64_t rows, int32_t d, int32_t rows_per_sample,
                              const float* scale_offset, float eps, void* out, int32_t out_dtype, void* stream) {
  return cond_layernorm(x, nullptr, rows, d, rows_per_sample, nullptr, scale_offset, eps, out, out_dtype, stream);
}

fwn_status fwn_cond_layernorm_residual(float* x, const void* residual, int64_t rows, int32_t d, int32_t rows_per_sample,
                                       const int32_t* out_node, const float* scale_offset, float eps, void* out,
                                       int32_t out_dtype, void* stream) {
  if (rows > 0 && !residual) return fail(FWN_ERR_INVALID_ARGUMENT, "null residual");
  return cond_layernorm(x, x, rows, d, rows_per_sample, out_node, scale_offset, eps, out, out_dtype, stream, residual);
}

fwn_status fwn_cond_layernorm_add(const float* x, const void* residual, float* x_out, int64_t rows, int32_t d,
                                  int32_t rows_per_sample, const float* scale_offset, float eps, void* out,
                                  int32_t out_dtype, void* stream) {
  if (rows > 0 && !residual) return fail(FWN_ERR_INVALID_ARGUMENT, "null residual");
  return cond_layernorm(x, x_out, rows, d, rows_per_sample, nullptr, scale_offset, eps, out, out_dtype, stream,
                        residual);
}

fwn_status fwn_cond_layernorm_scatter(const float* x, int64_t rows, int32_t d, int32_t rows_per_sample,
                                      const int32_t* out_node, const float* scale_offset, float eps, void* out,
                                      int32_t out_dtype, void* stream) {
  if (rows > 0 && !out_node) return fail(FWN_ERR_INVALID_ARGUMENT, "null out_node");
  return cond_layernorm(x, nullptr, rows, d, rows_per_sample, out_node, scale_offset, eps, out, out_dtype, stream);
}

size_t fwn_cond_layernorm_bwd_workspace(int64_t rows, int32_t d, int32_t rows_per_sample) {
  if (rows <= 0 || rows_per_sample <= 0 || d <= 0) return 0;
  return fwn::cond_layernorm_bwd_workspace(rows, d, rows_per_sample);
}

fwn_status fwn_cond_layernorm_bwd(const float* x, int64_t rows, int32_t d, int32_t rows_per_sample,
                                  const float* scale_offset, float eps, const void* dy, int32_t dy_dtype,
                                  const float* dx_in, float* dx, void* dx_bf16, float* dscale_offset, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  if (rows < 0 || rows_per_sample <= 0 || !(eps > 0.f))
    return fail(FWN_ERR_INVALID_ARGUMENT, "bad rows=%lld, rows_per_sample=%d or eps", static_cast<long long>(rows),
                rows_per_sample);
  if (d != 128 && d != 256 && d != 512) return fail(FWN_ERR_UNSUPPORTED, "d=%d not built for the backward", d);
  if (dy_dtype != FWN_DTYPE_BF16 && dy_dtype != FWN_DTYPE_F32)
    return fail(FWN_ERR_INVALID_ARGUMENT, "unknown dy dtype %d", dy_dtype);
  if (rows % rows_per_sample != 0)
    return fail(FWN_ERR_INVALID_ARGUMENT, "rows=%lld is not a multiple of rows_per_sample=%d",
                static_cast<long long>(rows), rows_per_sample);
  if (rows == 0) return ok();
  if (!x || !scale_offset || !dy || !dx || !dscale_offset || !workspace)
    return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  if (!aligned16(x) || !aligned16(scale_offset) || !aligned16(dy) || !aligned16(dx) ||
      (dx_in && !aligned16(dx_in)) || (dx_bf16 && !aligned16(dx_bf16)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const size_t need = fwn::cond_layernorm_bwd_workspace(rows, d, rows_per_sample);
  if (workspace_bytes < need)
    return fail(FWN_ERR_INVALID_ARGUMENT, "workspace of %zu bytes, %zu needed", workspace_bytes, need);
  cudaError_t e = fwn::launch_cond_layernorm_bwd(x, rows, d, rows_per_sample, scale_offset, eps, dy,
                                                 dy_dtype == FWN_DTYPE_BF16, dx_in, dx, dx_bf16, dscale_offset,
                                                 workspace, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cond_layernorm_bwd");
  return ok();
}

namespace {

// 2D map over a row-major bf16 matrix [rows, cols] (cols contiguous): box = 64 columns (128 bytes) x box_rows rows,
// 128-byte swizzle (the K-major operand layout of the GEMM).
// box_cols 64 with the 128-byte swizzle (GEMM operands) or 32 with the 64-byte swizzle (GEMM output chunks).
fwn_status make_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows, int box_cols = 64) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return fail(FWN_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FWN_ERR_INVALID_ARGUMENT, "cuTensorMapEncodeTiled (2d) failed (%d)", static_cast<int>(r));
  return FWN_OK;
}

}  // namespace

namespace {

// act: the public FWN_ACT_* value, or kGemmGatherAdd (the gathered-add epilogue, whose fields `adds` carries).
constexpr int32_t kGemmGatherAdd = 5;

fwn_status gemm_bf16(const void* a, const void* bt, const void* bias, void* c, void* aux, int64_t m, int32_t n,
                     int32_t k, int32_t act, void* stream, const fwn::GemmParams* adds = nullptr) {
  using C = fwn::GemmCfg;
  if (m <= 0 || n <= 0 || k <= 0) return fail(FWN_ERR_INVALID_ARGUMENT, "bad shape m=%lld n=%d k=%d", static_cast<long long>(m), n, k);
  if (n % C::BN != 0 || k % C::BK != 0)
    return fail(FWN_ERR_UNSUPPORTED, "n=%d must be a multiple of %d and k=%d of %d", n, C::BN, k, C::BK);
  if (!a || !bt || !c) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  const bool uses_aux = act == FWN_ACT_GELU_TANH_AUX || act == FWN_ACT_GELU_TANH_GRAD;
  if (uses_aux && !aux) return fail(FWN_ERR_INVALID_ARGUMENT, "activation %d needs the aux tensor", act);
  if (!aligned16(a) || !aligned16(bt) || !aligned16(c) || (bias && !aligned16(bias)) || (uses_aux && !aligned16(aux)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "pointers must be 16-byte aligned");
  const int64_t m_tiles = (m + C::BM - 1) / C::BM;
  if (m_tiles * (n / C::BN) >= (int64_t(1) << 31)) return fail(FWN_ERR_UNSUPPORTED, "m=%lld too large", static_cast<long long>(m));
  CUtensorMap ta, tb, tc, taux;
  fwn_status s;
  if ((s = make_map_2d(&ta, a, m, k, C::BM)) != FWN_OK) return s;
  if ((s = make_map_2d(&tb, bt, n, k, C::BN)) != FWN_OK) return s;
  if ((s = make_map_2d(&tc, c, m, n, 32, 32)) != FWN_OK) return s;
  taux = tc;
  if (uses_aux && (s = make_map_2d(&taux, aux, m, n, 32, 32)) != FWN_OK) return s;
  fwn::GemmParams p{};
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.c = static_cast<__nv_bfloat16*>(c);
  p.aux_in = act == FWN_ACT_GELU_TANH_GRAD ? static_cast<const __nv_bfloat16*>(aux) : nullptr;
  if (adds != nullptr) {
    p.add0 = adds->add0;
    p.idx0 = adds->idx0;
    p.rows0 = adds->rows0;
    p.add1 = adds->add1;
    p.idx1 = adds->idx1;
    p.rows1 = adds->rows1;
    p.swish = adds->swish;
  }
  p.m = m;
  p.n = n;
  p.k = k;
  p.act = act;
  p.n_tiles = n / C::BN;
  p.num_tiles = static_cast<int>(m_tiles * p.n_tiles);
  auto kernel = act == FWN_ACT_GELU_TANH        ? fwn::gemm_bf16_kernel<FWN_ACT_GELU_TANH>
                : act == FWN_ACT_GELU_TANH_AUX  ? fwn::gemm_bf16_kernel<FWN_ACT_GELU_TANH_AUX>
                : act == FWN_ACT_GELU_TANH_GRAD ? fwn::gemm_bf16_kernel<FWN_ACT_GELU_TANH_GRAD>
                : act == kGemmGatherAdd         ? fwn::gemm_bf16_kernel<kGemmGatherAdd>
                                                : fwn::gemm_bf16_kernel<FWN_ACT_NONE>;
  const int smem = act == FWN_ACT_GELU_TANH_GRAD ? fwn::GemmCfgT<FWN_ACT_GELU_TANH_GRAD>::SMEM_BYTES : C::SMEM_BYTES;
  int grid = 0;
  if ((s = persistent_grid(kernel, C::THREADS, smem, C::TMEM_COLS, p.num_tiles, &grid)) != FWN_OK) return s;
  kernel<<<grid, C::THREADS, smem, static_cast<cudaStream_t>(stream)>>>(ta, tb, tc, taux, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm launch");
  return ok();
}

}  // namespace

fwn_status fwn_gemm_bf16(const void* a, const void* bt, const void* bias, void* c, int64_t m, int32_t n, int32_t k,
                         int32_t act, void* stream) {
  if (act != FWN_ACT_NONE && act != FWN_ACT_GELU_TANH) return fail(FWN_ERR_INVALID_ARGUMENT, "unknown activation %d", act);
  return gemm_bf16(a, bt, bias, c, nullptr, m, n, k, act, stream);
}

fwn_status fwn_gemm_bf16_aux(const void* a, const void* bt, const void* bias, void* c, void* aux, int64_t m, int32_t n,
                             int32_t k, int32_t act, void* stream) {
  if (act != FWN_ACT_NONE && act != FWN_ACT_GELU_TANH && act != FWN_ACT_GELU_TANH_AUX && act != FWN_ACT_GELU_TANH_GRAD)
    return fail(FWN_ERR_INVALID_ARGUMENT, "unknown activation %d", act);
  return gemm_bf16(a, bt, bias, c, aux, m, n, k, act, stream);
}

fwn_status fwn_gemm_bf16_gather(const void* a, const void* bt, const void* bias, void* c, const void* add0,
                                const int32_t* idx0, int64_t rows0, const void* add1, const int32_t* idx1,
                                int64_t rows1, int64_t m, int32_t n, int32_t k, int32_t act, void* stream) {
  if (act != FWN_ACT_NONE && act != FWN_ACT_SWISH) return fail(FWN_ERR_INVALID_ARGUMENT, "unknown activation %d", act);
  if ((add0 && (!aligned16(add0) || rows0 <= 0)) || (add1 && (!aligned16(add1) || rows1 <= 0)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "added tensors must be 16-byte aligned with a positive row count");
  if ((add0 && !idx0 && rows0 < m) || (add1 && !idx1 && rows1 < m))
    return fail(FWN_ERR_INVALID_ARGUMENT, "an added tensor without an index needs m rows");
  fwn::GemmParams adds{};
  adds.add0 = static_cast<const __nv_bfloat16*>(add0);
  adds.idx0 = add0 ? idx0 : nullptr;
  adds.rows0 = rows0;
  adds.add1 = static_cast<const __nv_bfloat16*>(add1);
  adds.idx1 = add1 ? idx1 : nullptr;
  adds.rows1 = rows1;
  adds.swish = act == FWN_ACT_SWISH;
  return gemm_bf16(a, bt, bias, c, nullptr, m, n, k, kGemmGatherAdd, stream, &adds);
}

fwn_status fwn_gnn_gather_add_act(const void* e_proj, const void* s_proj, const int32_t* senders, const void* r_proj,
                                  const int32_t* receivers, const void* bias, int64_t rows, int32_t h, int32_t act,
                                  void* out, void* stream) {
  if (rows < 0 || h <= 0 || h % 8 != 0) return fail(FWN_ERR_INVALID_ARGUMENT, "bad rows=%lld or h=%d (a multiple of 8)",
                                                    static_cast<long long>(rows), h);
  if (act != FWN_ACT_NONE && act != FWN_ACT_SWISH) return fail(FWN_ERR_INVALID_ARGUMENT, "unknown activation %d", act);
  if (rows > 0 && !out) return fail(FWN_ERR_INVALID_ARGUMENT, "null out");
  for (const void* ptr : {e_proj, s_proj, r_proj, bias, static_cast<const void*>(out)})
    if (ptr && !aligned16(ptr)) return fail(FWN_ERR_INVALID_ARGUMENT, "operands must be 16-byte aligned");
  cudaError_t e = fwn::launch_gather_add_act(e_proj, s_proj, senders, r_proj, receivers, bias, rows, h,
                                             act == FWN_ACT_SWISH, out,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "gather_add_act");
  return ok();
}

fwn_status fwn_gnn_ln_segment_sum(const void* m, const int32_t* seg_ptr, int64_t n_out, int32_t f, const void* gamma,
                                  const void* beta, float eps, float norm, const float* residual, void* out,
                                  int32_t out_dtype, void* stream) {
  if (n_out < 0 || !(eps > 0.f)) return fail(FWN_ERR_INVALID_ARGUMENT, "bad n_out=%lld or eps", static_cast<long long>(n_out));
  if (f != 256 && f != 512 && f != 1024) return fail(FWN_ERR_UNSUPPORTED, "f=%d not built (256, 512, 1024)", f);
  if (out_dtype != FWN_DTYPE_BF16 && out_dtype != FWN_DTYPE_F32)
    return fail(FWN_ERR_INVALID_ARGUMENT, "unknown out dtype %d", out_dtype);
  if (n_out > 0 && (!m || !gamma || !beta || !out)) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  for (const void* ptr : {m, gamma, beta, static_cast<const void*>(residual), static_cast<const void*>(out)})
    if (ptr && !aligned16(ptr)) return fail(FWN_ERR_INVALID_ARGUMENT, "operands must be 16-byte aligned");
  cudaError_t e = fwn::launch_ln_segment_sum(m, seg_ptr, n_out, f, gamma, beta, eps, norm, residual, out,
                                             out_dtype == FWN_DTYPE_BF16, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "ln_segment_sum");
  return ok();
}

int32_t fwn_bitset_words(int32_t n_cols) { return n_cols > 0 ? fwn::bitset_words(n_cols) : 0; }

namespace {

fwn_status khop_common(const int32_t* indptr, const int32_t* indices, int32_t n, int32_t hops, uint32_t* reach,
                       uint32_t* scratch, void* stream, bool include_self) {
  if (n < 0 || hops < 0 || hops > 4096) return fail(FWN_ERR_INVALID_ARGUMENT, "bad n=%d or hops=%d", n, hops);
  if (n > 0 && (!indptr || !reach || !scratch)) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  if (n > 0 && (!aligned16(reach) || !aligned16(scratch)))
    return fail(FWN_ERR_INVALID_ARGUMENT, "reach and scratch must be 16-byte aligned");
  cudaError_t e = fwn::launch_khop(indptr, indices, n, hops, reach, scratch, static_cast<cudaStream_t>(stream),
                                   include_self);
  if (e != cudaSuccess) return cuda_fail(e, include_self ? "khop" : "walks");
  return ok();
}

}  // namespace

fwn_status fwn_khop_bitset(const int32_t* indptr, const int32_t* indices, int32_t n, int32_t hops, uint32_t* reach,
                           uint32_t* scratch, void* stream) {
  return khop_common(indptr, indices, n, hops, reach, scratch, stream, true);
}

fwn_status fwn_walk_bitset(const int32_t* indptr, const int32_t* indices, int32_t n, int32_t length, uint32_t* reach,
                           uint32_t* scratch, void* stream) {
  return khop_common(indptr, indices, n, length, reach, scratch, stream, false);
}

fwn_status fwn_bitset_csr_count(const uint32_t* bits, int32_t n_rows, int32_t n_cols, int32_t* indptr, void* ws,
                                size_t ws_bytes, void* stream) {
  if (n_rows < 0 || n_cols < 0) return fail(FWN_ERR_INVALID_ARGUMENT, "bad shape %d x %d", n_rows, n_cols);
  if (static_cast<int64_t>(n_rows) * n_cols >= (int64_t(1) << 31))
    return fail(FWN_ERR_UNSUPPORTED, "%d x %d mask: nnz may not fit int32", n_rows, n_cols);
  if (!indptr || (n_rows > 0 && !bits)) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  const size_t need = static_cast<size_t>(n_rows) * 4;
  if (n_rows > 0 && (!ws || ws_bytes < need)) return fail(FWN_ERR_WORKSPACE, "workspace of %zu bytes needed", need);
  cudaError_t e = fwn::launch_bitset_csr_count(bits, n_rows, n_cols, indptr, static_cast<int32_t*>(ws),
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bitset_csr_count");
  return ok();
}

fwn_status fwn_bitset_csr_fill(const uint32_t* bits, int32_t n_rows, int32_t n_cols, const int32_t* indptr,
                               int32_t* indices, void* stream) {
  if (n_rows < 0 || n_cols < 0) return fail(FWN_ERR_INVALID_ARGUMENT, "bad shape %d x %d", n_rows, n_cols);
  if (n_rows > 0 && (!bits || !indptr)) return fail(FWN_ERR_INVALID_ARGUMENT, "null pointer");
  cudaError_t e = fwn::launch_bitset_csr_fill(bits, n_rows, n_cols, indptr, indices, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "bitset_csr_fill");
  return ok();
}

fwn_status fwn_attn_fwd(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                        const fwn_tile_list* tiles, void* o, float* lse, void* stream) {
  fwn_status s = check_desc(desc);
  if (s != FWN_OK) return s;
  if ((s = check_tiles(tiles, desc, "tiles")) != FWN_OK) return s;
  if (!q || !k || !v || !o) return fail(FWN_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(FWN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const fwn_attn_desc& d = *desc;
  int layout = 0;
  if (tiles->cols) {
    layout = gather_layout(d, false);
    if (layout < 0) return fail(FWN_ERR_INVALID_ARGUMENT, "gathered lists need a node-major or head-major packed layout");
  }
  const bool g = tiles->cols != nullptr;
  if (use_wide(d, *tiles))
    return d.head_dim == 64 ? launch_fwd_wide<64>(d, q, k, v, *tiles, o, lse, st)
                            : launch_fwd_wide<128>(d, q, k, v, *tiles, o, lse, st);
  if (d.mode == FWN_MODE_BF16) {
    if (d.head_dim == 64)
      return g ? launch_fwd<64, false, true>(d, q, k, v, *tiles, o, lse, layout, st)
               : launch_fwd<64, false, false>(d, q, k, v, *tiles, o, lse, layout, st);
    return g ? launch_fwd<128, false, true>(d, q, k, v, *tiles, o, lse, layout, st)
             : launch_fwd<128, false, false>(d, q, k, v, *tiles, o, lse, layout, st);
  }
  if (d.mode == FWN_MODE_TF32 && d.head_dim == 64)
    return g ? launch_fwd<64, true, true>(d, q, k, v, *tiles, o, lse, layout, st)
             : launch_fwd<64, true, false>(d, q, k, v, *tiles, o, lse, layout, st);
  if (d.mode == FWN_MODE_TF32)
    return g ? launch_fwd<128, true, true>(d, q, k, v, *tiles, o, lse, layout, st)
             : launch_fwd<128, true, false>(d, q, k, v, *tiles, o, lse, layout, st);
  if (d.mode == FWN_MODE_TF32X3 && d.head_dim == 64)
    return g ? launch_fwd<64, true, true, true>(d, q, k, v, *tiles, o, lse, layout, st)
             : launch_fwd<64, true, false, true>(d, q, k, v, *tiles, o, lse, layout, st);
  return g ? launch_fwd<128, true, true, true>(d, q, k, v, *tiles, o, lse, layout, st)
           : launch_fwd<128, true, false, true>(d, q, k, v, *tiles, o, lse, layout, st);
}

fwn_status fwn_test_attn_fwd_timeout(const fwn_attn_desc* desc, const void* q, const void* k, const void* v,
                                     const fwn_tile_list* tiles, void* o, float* lse, uint64_t wait_limit_ns,
                                     void* stream) {
  fwn_status s = check_desc(desc);
  if (s != FWN_OK) return s;
  if ((s = check_tiles(tiles, desc, "tiles")) != FWN_OK) return s;
  if (!q || !k || !v || !o) return fail(FWN_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o))
    return fail(FWN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  if (wait_limit_ns < 100000ull || wait_limit_ns > fwn::kWaitLimitNs)
    return fail(FWN_ERR_INVALID_ARGUMENT, "wait_limit_ns must lie in [1e5, %llu]", fwn::kWaitLimitNs);
  const fwn_attn_desc& d = *desc;
  if (d.mode != FWN_MODE_BF16 || d.head_dim != 64 || use_wide(d, *tiles))
    return fail(FWN_ERR_UNSUPPORTED, "the timeout test runs the narrow bf16 head_dim-64 forward only");
  int layout = 0;
  if (tiles->cols) {
    layout = gather_layout(d, false);
    if (layout < 0) return fail(FWN_ERR_INVALID_ARGUMENT, "gathered lists need a node-major or head-major packed layout");
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  return tiles->cols ? launch_fwd<64, false, true>(d, q, k, v, *tiles, o, lse, layout, st, wait_limit_ns, 1)
                     : launch_fwd<64, false, false>(d, q, k, v, *tiles, o, lse, layout, st, wait_limit_ns, 1);
}

fwn_status fwn_attn_bwd_workspace_size(const fwn_attn_desc* desc, size_t* bytes) {
  fwn_status s = check_desc(desc);
  if (s != FWN_OK) return s;
  if (!bytes) return fail(FWN_ERR_INVALID_ARGUMENT, "bytes is null");
  *bytes = static_cast<size_t>(desc->batch) * desc->heads * fwn_lse_rows(desc->n) * sizeof(float);
  return ok();
}

fwn_status fwn_attn_bwd(const fwn_attn_desc* desc, const void* q, const void* k, const void* v, const void* o,
                        const float* lse, const void* d_o, const fwn_tile_list* tiles, const fwn_tile_list* tiles_t,
                        void* dq, void* dk, void* dv, void* ws, size_t ws_bytes, void* stream) {
  return bwd_dispatch(desc, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, ws, ws_bytes, kAll, stream);
}

fwn_status fwn_attn_bwd_delta(const fwn_attn_desc* desc, const void* o, const void* d_o, void* ws, size_t ws_bytes,
                              void* stream) {
  return bwd_dispatch(desc, nullptr, nullptr, nullptr, o, nullptr, d_o, nullptr, nullptr, nullptr, nullptr, nullptr, ws,
                      ws_bytes, kDelta, stream);
}

fwn_status fwn_attn_bwd_dq(const fwn_attn_desc* desc, const void* q, const void* k, const void* v, const float* lse,
                           const void* d_o, const fwn_tile_list* tiles, void* dq, const void* ws, size_t ws_bytes,
                           void* stream) {
  return bwd_dispatch(desc, q, k, v, nullptr, lse, d_o, tiles, nullptr, dq, nullptr, nullptr, ws, ws_bytes, kDq, stream);
}

fwn_status fwn_attn_bwd_dkv(const fwn_attn_desc* desc, const void* q, const void* k, const void* v, const float* lse,
                            const void* d_o, const fwn_tile_list* tiles_t, void* dk, void* dv, const void* ws,
                            size_t ws_bytes, void* stream) {
  return bwd_dispatch(desc, q, k, v, nullptr, lse, d_o, nullptr, tiles_t, nullptr, dk, dv, ws, ws_bytes, kDkv, stream);
}

fwn_status fwn_attn_bwd_noalloc(const fwn_attn_desc* desc, const void* q, const void* k, const void* v, const void* o,
                                const float* lse, const void* d_o, const fwn_tile_list* tiles,
                                const fwn_tile_list* tiles_t, void* dq, void* dk, void* dv, void* stream) {
  fwn_status s = check_desc(desc);
  if (s != FWN_OK) return s;
  const long long rows = static_cast<long long>(desc->batch) * desc->heads * fwn_lse_rows(desc->n);
  if (rows > FWN_NOALLOC_DELTA_ROWS)
    return fail(FWN_ERR_WORKSPACE,
                "fwn_attn_bwd_noalloc: batch * heads * lse_rows = %lld exceeds its fixed capacity of %d rows; "
                "use fwn_attn_bwd with a workspace",
                rows, FWN_NOALLOC_DELTA_ROWS);
  float* delta = nullptr;
  if ((s = noalloc_delta(&delta)) != FWN_OK) return s;
  return bwd_dispatch(desc, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta,
                      static_cast<size_t>(FWN_NOALLOC_DELTA_ROWS) * sizeof(float), kAll, stream);
}

#ifdef FWN_TRACE
FWN_API int fwn_trace_dump(unsigned long long* host, int words) {
  const int n = fwn::kTraceCtas * fwn::kTraceEvents;
  cudaDeviceSynchronize();
  cudaMemcpy(host, trace_buffer_peek(), sizeof(unsigned long long) * (words < n ? words : n), cudaMemcpyDeviceToHost);
  return n;
}
#endif

}  // extern "C"

namespace {

fwn_status bwd_dispatch(const fwn_attn_desc* desc, const void* q, const void* k, const void* v, const void* o,
                        const float* lse, const void* d_o, const fwn_tile_list* tiles, const fwn_tile_list* tiles_t,
                        void* dq, void* dk, void* dv, const void* ws, size_t ws_bytes, int parts, void* stream) {
  fwn_status s = check_desc(desc);
  if (s != FWN_OK) return s;
  if ((parts & kDq) && (s = check_tiles(tiles, desc, "tiles")) != FWN_OK) return s;
  if ((parts & kDkv) && (s = check_tiles(tiles_t, desc, "tiles_t")) != FWN_OK) return s;
  const void* need_ptrs[] = {(parts & kDelta) ? o : d_o, d_o, (parts & (kDq | kDkv)) ? q : d_o,
                             (parts & (kDq | kDkv)) ? k : d_o, (parts & (kDq | kDkv)) ? v : d_o,
                             (parts & (kDq | kDkv)) ? static_cast<const void*>(lse) : d_o, (parts & kDq) ? dq : d_o,
                             (parts & kDkv) ? dk : d_o, (parts & kDkv) ? dv : d_o};
  for (const void* ptr : need_ptrs) {
    if (!ptr) return fail(FWN_ERR_INVALID_ARGUMENT, "null tensor pointer");
    if (!aligned16(ptr)) return fail(FWN_ERR_INVALID_ARGUMENT, "tensors must be 16-byte aligned");
  }
  size_t need = 0;
  fwn_attn_bwd_workspace_size(desc, &need);
  if (!ws || ws_bytes < need || !aligned16(ws))
    return fail(FWN_ERR_WORKSPACE, "workspace of %zu bytes (16-byte aligned) needed", need);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const fwn_attn_desc d = resolve_grad_strides(desc);
  float* delta = static_cast<float*>(const_cast<void*>(ws));
  if (d.mode == FWN_MODE_BF16) {
    if (d.head_dim == 64) return launch_bwd<64, false>(d, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta, parts, st);
    return launch_bwd<128, false>(d, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta, parts, st);
  }
  if (d.mode == FWN_MODE_TF32 && d.head_dim == 64)
    return launch_bwd<64, true>(d, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta, parts, st);
  if (d.mode == FWN_MODE_TF32)
    return launch_bwd<128, true>(d, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta, parts, st);
  if (d.mode == FWN_MODE_TF32X3 && d.head_dim == 64)
    return launch_bwd<64, true, true>(d, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta, parts, st);
  return launch_bwd<128, true, true>(d, q, k, v, o, lse, d_o, tiles, tiles_t, dq, dk, dv, delta, parts, st);
}

}  // namespace
