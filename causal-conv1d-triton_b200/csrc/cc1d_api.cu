// C ABI of the causal depthwise conv1d library: argument checks, path selection (TMA kernels for
// widths 2..16 on 16-byte-aligned layouts, their plain-load / cp.async variants on layouts with
// 8-byte rows, generic kernels otherwise), tensor-map encoding, grid
// sizing from the measured occupancy and SM count, and the T == 0 cases. Declared in
// include/causal_conv1d_b200.h, where each entry point names the reference launch it replaces.
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "causal_conv1d_b200.h"
#include "cc1d_dispatch.h"
#include "cc1d_reduce_kernels.cuh"
#include "cc1d_seqidx_kernel.cuh"
#include "cc1d_update_kernel.cuh"
#include "cc1d_copy_kernel.cuh"

namespace cc1d {

static_assert(kMaxDoutPieces == CC1D_MAX_DOUT_PIECES, "one limit on dout pieces");

__device__ unsigned g_status_word;

namespace {

thread_local int t_last_cuda_error = 0;

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = static_cast<int>(e);
  return CC1D_ERR_CUDA;
}

#define CC1D_TRY_CUDA(call)                    \
  do {                                         \
    const cudaError_t e_ = (call);             \
    if (e_ != cudaSuccess) return cuda_fail(e_); \
  } while (0)

#define CC1D_TRY(call)        \
  do {                        \
    const int r_ = (call);    \
    if (r_ != CC1D_OK) return r_; \
  } while (0)

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  int sms = 0;
  unsigned* status = nullptr;  // device address of g_status_word on this device
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
bool g_dev_ready[kMaxDevices] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::map<std::tuple<const void*, int, int>, int> g_occupancy;  // (fn, device, smem) -> CTAs/SM
std::map<std::pair<const void*, int>, int> g_smem_attr;         // (fn, device) -> max dyn smem set

int elem_size(int dtype) { return dtype == kF32 ? 4 : 2; }
bool valid_dtype(int dtype) { return dtype == kF32 || dtype == kF16 || dtype == kBF16; }
int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

int device_info(DeviceInfo* out, int* dev_out) {
  int dev = 0;
  CC1D_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return CC1D_ERR_INVALID;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_ready[dev]) {
    int sms = 0;
    CC1D_TRY_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    void* st = nullptr;
    CC1D_TRY_CUDA(cudaGetSymbolAddress(&st, g_status_word));
    g_dev[dev].sms = sms;
    g_dev[dev].status = static_cast<unsigned*>(st);
    g_dev_ready[dev] = true;
  }
  *out = g_dev[dev];
  *dev_out = dev;
  return CC1D_OK;
}

// CTAs of `k` that fit on one SM with k.smem bytes of dynamic shared memory. The function's
// dynamic shared memory limit is raised to `max_smem` once per device.
int occupancy(const KernelInfo& k, int max_smem, int dev, int* occ) {
  std::lock_guard<std::mutex> lk(g_mu);
  const auto key = std::make_tuple(k.fn, dev, k.smem);
  auto it = g_occupancy.find(key);
  if (it != g_occupancy.end()) {
    *occ = it->second;
    return CC1D_OK;
  }
  const auto akey = std::make_pair(k.fn, dev);
  auto at = g_smem_attr.find(akey);
  if (at == g_smem_attr.end() || at->second < max_smem) {
    CC1D_TRY_CUDA(cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem));
    g_smem_attr[akey] = max_smem;
  }
  int n = 0;
  CC1D_TRY_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k.fn, k.threads, k.smem));
  if (n < 1) return CC1D_ERR_UNSUPPORTED;
  g_occupancy[key] = n;
  *occ = n;
  return CC1D_OK;
}

int tensor_map_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    CC1D_TRY_CUDA(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || p == nullptr) return cuda_fail(cudaErrorSymbolNotFound);
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  *fn = g_encode;
  return CC1D_OK;
}

// Whether a (B, T, D) channels-last tensor at `ptr` with batch/time strides (in elements) can be
// read by the TMA kernels: 16-byte aligned base and strides, and rows of out/dx (D elements)
// that are whole 16-byte vectors.
// The backward walk's plain mode copies 8-byte chunks: base, strides and rows 8-byte multiples.
bool chunk_layout_ok(const void* ptr, int64_t sb, int64_t st, int64_t B, int64_t D, int es) {
  if (reinterpret_cast<uintptr_t>(ptr) % 8 != 0) return false;
  if (st <= 0 || (st * es) % 8 != 0) return false;
  if (B > 1 && (sb <= 0 || (sb * es) % 8 != 0)) return false;
  return (D * es) % 8 == 0;
}

bool tma_layout_ok(const void* ptr, int64_t sb, int64_t st, int64_t B, int64_t D, int es) {
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0) return false;
  if (st <= 0 || (st * es) % 16 != 0) return false;
  if (B > 1 && (sb <= 0 || (sb * es) % 16 != 0)) return false;
  return (D * es) % 16 == 0;
}

// 3-D tensor map over a (B, T, D) channels-last tensor, as dims (D, T, B), box (box_d, box_t, 1).
// Rows outside [0, T) and channels outside [0, D) read as zero.
bool encode_3d_uncached(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t T, int64_t D, int64_t sb,
                        int64_t st, int box_d, int box_t) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
  if (tensor_map_encoder(&enc) != CC1D_OK) return false;
  const int es = elem_size(dtype);
  const CUtensorMapDataType dt = dtype == kF32   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : dtype == kF16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(T), static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(st * es),
                                 static_cast<cuuint64_t>(B > 1 ? sb * es : T * st * es)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_d), static_cast<cuuint32_t>(box_t), 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  const CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The encoded maps of recent calls, keyed by every argument of the encoding (the map is a pure
// function of them): a training loop passes the same buffers step after step, and re-encoding
// two or three maps per call is a measurable share of a small call's host time.
struct MapKey {
  const void* base;
  int64_t B, T, D, sb, st;
  int dtype, box_d, box_t;
  bool operator==(const MapKey& o) const {
    return base == o.base && B == o.B && T == o.T && D == o.D && sb == o.sb && st == o.st && dtype == o.dtype &&
           box_d == o.box_d && box_t == o.box_t;
  }
};
constexpr int kMapCache = 64;
struct MapEntry {
  MapKey key;
  CUtensorMap map;
  bool used = false;
};
MapEntry g_maps[kMapCache];
int g_map_next = 0;

bool encode_3d(CUtensorMap* map, const void* base, int dtype, int64_t B, int64_t T, int64_t D, int64_t sb,
               int64_t st, int box_d, int box_t) {
  const MapKey key{base, B, T, D, sb, st, dtype, box_d, box_t};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    for (const MapEntry& e : g_maps) {
      if (e.used && e.key == key) {
        *map = e.map;
        return true;
      }
    }
  }
  if (!encode_3d_uncached(map, base, dtype, B, T, D, sb, st, box_d, box_t)) return false;
  std::lock_guard<std::mutex> lk(g_mu);
  MapEntry& e = g_maps[g_map_next];
  g_map_next = (g_map_next + 1) % kMapCache;
  e.key = key;
  e.map = *map;
  e.used = true;
  return true;
}

// Template width of the TMA kernels for a true width W, or 0 for the generic path. Widths 9..16
// run on the width-12 or width-16 kernels with leading zero taps (identical results).
int tma_width(int64_t W) {
  if (W <= 8) return static_cast<int>(W);
  if (W <= 12) return 12;
  if (W <= 16) return 16;
  return 0;
}

KernelInfo fwd_tma_for(int dtype, int W, bool seq, bool silu, bool plain) {
  if (dtype == kBF16) return fwd_tma_info<__nv_bfloat16>(W, seq, silu, plain);
  if (dtype == kF16) return fwd_tma_info<__half>(W, seq, silu, plain);
  return fwd_tma_info<float>(W, seq, silu, plain);
}
KernelInfo bwd_tma_for(int dtype, int W, bool seq, bool silu, bool plain, bool long_stages = false) {
  if (dtype == kBF16) return bwd_tma_info<__nv_bfloat16>(W, seq, silu, plain, long_stages);
  if (dtype == kF16) return bwd_tma_info<__half>(W, seq, silu, plain, long_stages);
  return bwd_tma_info<float>(W, seq, silu, plain, long_stages);
}
KernelInfo fwd_generic_for(int dtype, int W) {
  if (dtype == kBF16) return fwd_generic_info<__nv_bfloat16>(W);
  if (dtype == kF16) return fwd_generic_info<__half>(W);
  return fwd_generic_info<float>(W);
}
KernelInfo bwd_generic_for(int dtype, int W) {
  if (dtype == kBF16) return bwd_generic_info<__nv_bfloat16>(W);
  if (dtype == kF16) return bwd_generic_info<__half>(W);
  return bwd_generic_info<float>(W);
}

int launch_fill(void* dst, int dst_dtype, const void* src, int src_dtype, int64_t n, int sms, cudaStream_t stream) {
  if (n <= 0) return CC1D_OK;
  const int blocks = static_cast<int>(std::min<int64_t>(cdiv(n, 256), static_cast<int64_t>(sms) * 8));
  cc1d_fill_kernel<<<blocks, 256, 0, stream>>>(dst, dst_dtype, src, src_dtype, n);
  CC1D_TRY_CUDA(cudaGetLastError());
  return CC1D_OK;
}

int check_sizes(int64_t B, int64_t T, int64_t D, int64_t W) {
  if (B < 0 || T < 0 || D < 0 || W < 2) return CC1D_ERR_INVALID;
  if (B >= (int64_t(1) << 31) || T >= (int64_t(1) << 31) || D >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
  if (B * cdiv(T, 64) >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
  if (W > kGenericMaxWidth) return CC1D_ERR_UNSUPPORTED;
  return CC1D_OK;
}

// Launch plan of the backward: which kernel, how many CTAs, how many partial rows.
struct BwdPlan {
  bool tma = false;
  bool plain = false;  // TMA-path kernels with the stage copied by cp.async (see BwdWalkParams)
  int wt = 0;     // template width of the TMA kernels (0: generic path)
  KernelInfo k;
  int max_smem = 0;
  int P = 0;      // partial rows (CTAs per channel block / group)
  int n_blk = 0;  // channel blocks (generic) or channel groups (TMA)
  int n_tt = 0;   // generic: time tiles per batch row
  int64_t rows_per_part = 0;  // TMA: flattened (batch, time) rows per CTA
  int64_t grid = 0;
  int64_t ws_bytes = 0;
};

// Rows per CTA from which the backward's warp-specialized walk uses 24-row stages (measured on B200:
// 7282 rows per CTA 3 % faster, 2260 rows equal, 886 rows 7 % slower than with 16-row stages).
constexpr int64_t kLongWalkRows = 2048;

int plan_bwd_uncached(const void* x, int64_t sxb, int64_t sxt, const void* dy, int64_t syb, int64_t syt, int64_t B,
                      int64_t T, int64_t D, int64_t W, int x_dtype, bool seq, bool silu, const DeviceInfo& di, int dev,
                      BwdPlan* pl) {
  const int es = elem_size(x_dtype);
  pl->wt = tma_width(W);
  pl->tma = pl->wt > 0 && tma_layout_ok(x, sxb, sxt, B, D, es) && tma_layout_ok(dy, syb, syt, B, D, es);
  if (!pl->tma && pl->wt > 0 && chunk_layout_ok(x, sxb, sxt, B, D, es) && chunk_layout_ok(dy, syb, syt, B, D, es)) {
    pl->tma = true;
    pl->plain = true;
  }
  const int64_t rows = B * T;
  if (pl->tma) {
    // One resident wave per launch: P CTAs per channel group, each walking an equal stretch of the
    // B*T rows (a multiple of the stage height). The variants with and without seq_idx and SiLU
    // may differ in CTA width and occupancy (the SiLU kernels of widths 5..8 are warp-specialized,
    // one CTA of 1024 channels per SM); the workspace query sees neither flag, so the workspace is
    // sized for the largest partial count of the four, and each launch uses its own.
    int64_t p_max = 1;
    // Stretch of rows per CTA and partial count for one kernel variant.
    auto split = [&](const KernelInfo& kv, int64_t* rpp, int64_t* P) -> int {
      if (kv.fn == nullptr) return CC1D_ERR_INVALID;
      if (kv.min_regs > 0) {
        // A warp-specialized kernel moves registers between its warpgroups with setmaxnreg; the
        // increase waits until the registers exist, so the launch must hold the whole split.
        cudaFuncAttributes fa{};
        CC1D_TRY_CUDA(cudaFuncGetAttributes(&fa, kv.fn));
        if (fa.numRegs < kv.min_regs) return CC1D_ERR_UNSUPPORTED;
      }
      int o = 0;
      CC1D_TRY(occupancy(kv, kv.smem, dev, &o));
      const int64_t n_blk = cdiv(D, kv.d_tile);
      const int64_t rs = kv.t_tile;
      const int64_t cap = static_cast<int64_t>(di.sms) * o;
      const int64_t pw = std::max<int64_t>(1, std::min<int64_t>(cdiv(rows, rs), cap / n_blk));
      *rpp = cdiv(cdiv(rows, pw), rs) * rs;
      *P = cdiv(rows, *rpp);
      return CC1D_OK;
    };
    for (int v = 0; v < 4; ++v) {
      const bool vseq = (v & 1) != 0, vsilu = (v & 2) != 0;
      KernelInfo kv = bwd_tma_for(x_dtype, pl->wt, vseq, vsilu, pl->plain);
      int64_t rpp = 0, P = 0;
      CC1D_TRY(split(kv, &rpp, &P));
      // Walks of at least kLongWalkRows rows per CTA take the 24-row-stage kernel where there is
      // one (the warp-specialized layout); shorter ones keep 16-row stages, whose ring fills and
      // drains faster.
      if (rpp >= kLongWalkRows) {
        const KernelInfo kl = bwd_tma_for(x_dtype, pl->wt, vseq, vsilu, pl->plain, true);
        if (kl.fn != kv.fn) {
          kv = kl;
          CC1D_TRY(split(kv, &rpp, &P));
        }
      }
      const int64_t n_blk = cdiv(D, kv.d_tile);
      p_max = std::max(p_max, P);
      if (vseq == seq && vsilu == silu) {
        pl->k = kv;
        pl->max_smem = kv.smem;
        pl->n_blk = static_cast<int>(n_blk);
        pl->rows_per_part = rpp;
        pl->P = static_cast<int>(P);
      }
    }
    pl->grid = static_cast<int64_t>(pl->P) * pl->n_blk;
    if (pl->grid >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
    pl->ws_bytes = p_max * (W + 1) * D * 4;
    return CC1D_OK;
  }
  int occ = 0;
  pl->k = bwd_generic_for(x_dtype, static_cast<int>(W));
  pl->max_smem = generic_bwd_smem(kGenericMaxWidth);
  CC1D_TRY(occupancy(pl->k, pl->max_smem, dev, &occ));
  pl->n_blk = static_cast<int>(cdiv(D, pl->k.d_tile));
  const int64_t cap = static_cast<int64_t>(di.sms) * occ;
  pl->n_tt = static_cast<int>(cdiv(T, pl->k.t_tile));
  const int64_t M = B * pl->n_tt;
  pl->P = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(M, cap / pl->n_blk)));
  pl->grid = static_cast<int64_t>(pl->P) * pl->n_blk;
  if (pl->grid >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
  pl->ws_bytes = static_cast<int64_t>(pl->P) * (W + 1) * D * 4;
  return CC1D_OK;
}

// The plan depends on the sizes, the element type, the device, the kernel variant (seq_idx,
// activation) and on which layouts x and dout have (TMA, cp.async chunks, or neither), not on
// the addresses themselves: plans are cached by exactly those.
struct PlanKey {
  int64_t B, T, D, W;
  int x_dtype, dev, layout;
  bool seq, silu;
  bool operator<(const PlanKey& o) const {
    return std::tie(B, T, D, W, x_dtype, dev, layout, seq, silu) <
           std::tie(o.B, o.T, o.D, o.W, o.x_dtype, o.dev, o.layout, o.seq, o.silu);
  }
};
std::map<PlanKey, BwdPlan> g_plans;

int plan_bwd(const void* x, int64_t sxb, int64_t sxt, const void* dy, int64_t syb, int64_t syt, int64_t B, int64_t T,
             int64_t D, int64_t W, int x_dtype, bool seq, bool silu, const DeviceInfo& di, int dev, BwdPlan* pl) {
  const int es = elem_size(x_dtype);
  const int layout = (tma_layout_ok(x, sxb, sxt, B, D, es) && tma_layout_ok(dy, syb, syt, B, D, es))       ? 2
                     : (chunk_layout_ok(x, sxb, sxt, B, D, es) && chunk_layout_ok(dy, syb, syt, B, D, es)) ? 1
                                                                                                            : 0;
  const PlanKey key{B, T, D, W, x_dtype, dev, layout, seq, silu};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_plans.find(key);
    if (it != g_plans.end()) {
      *pl = it->second;
      return CC1D_OK;
    }
  }
  CC1D_TRY(plan_bwd_uncached(x, sxb, sxt, dy, syb, syt, B, T, D, W, x_dtype, seq, silu, di, dev, pl));
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_plans.size() > 4096) g_plans.clear();
  g_plans[key] = *pl;
  return CC1D_OK;
}

// Workspace bytes the backward of this problem needs (0 for an empty one), or the error code
// cc1d_bwd would return for the same sizes, dtype and device. The plan does not depend on
// seq_idx or the activation.
int workspace_need(const void* x, int64_t sxb, int64_t sxt, const void* dy, int64_t syb, int64_t syt, int64_t B,
                   int64_t T, int64_t D, int64_t W, int x_dtype, int64_t* bytes) {
  *bytes = 0;
  if (!valid_dtype(x_dtype)) return CC1D_ERR_INVALID;
  CC1D_TRY(check_sizes(B, T, D, W));
  if (B == 0 || D == 0 || T == 0) return CC1D_OK;
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  BwdPlan pl;
  CC1D_TRY(plan_bwd(x, sxb, sxt, dy, syb, syt, B, T, D, W, x_dtype, false, false, di, dev, &pl));
  *bytes = pl.ws_bytes;
  return CC1D_OK;
}

template <typename T>
const void* update_vec_for_width(int W) {
  switch (W) {
    case 2: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 2>);
    case 3: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 3>);
    case 4: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 4>);
    case 5: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 5>);
    case 6: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 6>);
    case 7: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 7>);
    case 8: return reinterpret_cast<const void*>(&cc1d_update_vec_kernel<T, 8>);
    default: return nullptr;
  }
}

// The vector decode kernel for x and state of one element type and widths 2..8, else null.
const void* update_vec_kernel(int x_dtype, int state_dtype, int W) {
  if (x_dtype != state_dtype) return nullptr;
  if (x_dtype == kBF16) return update_vec_for_width<__nv_bfloat16>(W);
  if (x_dtype == kF16) return update_vec_for_width<__half>(W);
  return update_vec_for_width<float>(W);
}

}  // namespace
}  // namespace cc1d

namespace cc1d {
namespace {

// The backward behind cc1d_bwd (one dout piece, contiguous dx) and cc1d_bwd_split (dout as channel
// pieces, dx at strides; TMA path required, else CC1D_ERR_LAYOUT before any device work).
int bwd_impl(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight, const void* bias,
             const void* initial_states, const int32_t* seq_idx, const cc1d_dout_piece* pieces, int n_pieces,
             const void* dfinal_states, void* dx, int64_t stride_dx_batch, int64_t stride_dx_time, void* dweight,
             void* dbias, void* dinit, float* grad_f32, void* workspace, int64_t workspace_bytes, int64_t batch,
             int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int weight_dtype, int bias_dtype,
             int init_dtype, int silu, void* stream_, bool split) {
  const void* dout = pieces[0].ptr;
  const int64_t stride_dout_batch = pieces[0].stride_batch, stride_dout_time = pieces[0].stride_time;
  if (!valid_dtype(x_dtype) || !valid_dtype(weight_dtype) || (bias && !valid_dtype(bias_dtype)) ||
      (initial_states && !valid_dtype(init_dtype)))
    return CC1D_ERR_INVALID;
  if (dinit != nullptr && initial_states == nullptr) return CC1D_ERR_INVALID;
  if (grad_f32 == nullptr && dweight == nullptr) return CC1D_ERR_INVALID;
  CC1D_TRY(check_sizes(batch, seqlen, dim, width));
  if (batch == 0 || dim == 0) return CC1D_OK;
  const int64_t B = batch, T = seqlen, D = dim, W = width, PAD = W - 1;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  if (T == 0) {  // dinit = dfinal (or zero); no output rows, so dweight = dbias = 0
    if (dinit) CC1D_TRY(launch_fill(dinit, init_dtype, dfinal_states, x_dtype, B * PAD * D, di.sms, stream));
    if (grad_f32) {
      CC1D_TRY(launch_fill(grad_f32, kF32, nullptr, kF32, (W + 1) * D, di.sms, stream));
    } else {
      CC1D_TRY(launch_fill(dweight, weight_dtype, nullptr, kF32, W * D, di.sms, stream));
      if (bias && dbias) CC1D_TRY(launch_fill(dbias, bias_dtype, nullptr, kF32, D, di.sms, stream));
    }
    return CC1D_OK;
  }
  if (!x || !weight || !dout || !dx) return CC1D_ERR_INVALID;

  BwdPlan pl;
  CC1D_TRY(plan_bwd(x, stride_x_batch, stride_x_time, dout, stride_dout_batch, stride_dout_time, B, T, D, W, x_dtype,
                    seq_idx != nullptr, silu != 0, di, dev, &pl));
  if (split) {
    // Every piece and dx must suit the TMA walk: piece boundaries on channel blocks, 16-byte
    // aligned bases and strides (dx is written as 8-byte vectors at these strides).
    const int es = elem_size(x_dtype);
    bool ok = pl.tma && !pl.plain && reinterpret_cast<uintptr_t>(dx) % 16 == 0 && stride_dx_time >= D &&
              (stride_dx_time * es) % 16 == 0 && (B == 1 || (stride_dx_batch * es) % 16 == 0);
    int64_t c0 = 0;
    for (int i = 0; ok && i < n_pieces; ++i) {
      ok = c0 % pl.k.box_d == 0 &&
           tma_layout_ok(pieces[i].ptr, pieces[i].stride_batch, pieces[i].stride_time, B, pieces[i].channels, es);
      c0 += pieces[i].channels;
    }
    if (!ok) return CC1D_ERR_LAYOUT;
  }
  if (workspace == nullptr || workspace_bytes < pl.ws_bytes) return CC1D_ERR_WORKSPACE;
  float* partials = static_cast<float*>(workspace);

  bool launched = false;
  if (pl.tma) {
    BwdWalkParams p{};
    const int PADi = pl.wt - 1;  // halo rows of the template width
    const int box_d = pl.k.box_d;  // one channel block per consumer warp
    // Plain mode (layout beyond a tensor map, see plan_bwd): no maps; the producer copies chunks.
    bool maps = pl.plain ||
                encode_3d(&p.tmap_x, x, x_dtype, B, T, D, stride_x_batch, stride_x_time, box_d, pl.k.t_tile + PADi);
    p.x = x, p.dy = pieces[0].ptr;
    p.sxb = stride_x_batch, p.sxt = stride_x_time;
    p.syb = pieces[0].stride_batch, p.syt = pieces[0].stride_time;
    int64_t c_end = 0;
    for (int i = 0; maps && i < n_pieces; ++i) {
      if (!pl.plain)
        maps = encode_3d(&p.tmap_dy[i], pieces[i].ptr, x_dtype, B, T, pieces[i].channels, pieces[i].stride_batch,
                         pieces[i].stride_time, box_d, pl.k.t_tile);
      c_end += pieces[i].channels;
      p.dy_end[i] = static_cast<int>(c_end);
    }
    p.n_dy = n_pieces;
    p.sdxb = stride_dx_batch, p.sdxt = stride_dx_time;
    if (!maps && split) return CC1D_ERR_LAYOUT;
    if (maps) {
      int occ = 0;
      CC1D_TRY(occupancy(pl.k, pl.max_smem, dev, &occ));
      p.weight = weight, p.bias = bias, p.init = initial_states, p.seq = seq_idx;
      p.dfinal = dfinal_states, p.dx = dx, p.dinit = dinit, p.partials = partials, p.status = di.status;
      p.rows_per_part = pl.rows_per_part;
      p.B = static_cast<int>(B), p.T = static_cast<int>(T), p.D = static_cast<int>(D), p.W = static_cast<int>(W);
      p.n_groups = pl.n_blk;
      p.w_dtype = weight_dtype, p.b_dtype = bias_dtype, p.init_dtype = init_dtype;
      void* args[] = {&p};
      CC1D_TRY_CUDA(
          cudaLaunchKernel(pl.k.fn, dim3(static_cast<unsigned>(pl.grid)), dim3(pl.k.threads), args, pl.k.smem, stream));
      launched = true;
    }
  }
  if (!launched) {
    if (split) return CC1D_ERR_LAYOUT;  // unreachable: the split call requires the TMA path
    // The tensor maps could not be encoded: re-plan on the generic path, whose partial count is
    // never larger than the TMA path's, so the workspace still suffices.
    if (pl.tma) {
      const int64_t ws_tma = pl.ws_bytes;
      pl.tma = false;
      pl.k = bwd_generic_for(x_dtype, static_cast<int>(W));
      pl.max_smem = generic_bwd_smem(kGenericMaxWidth);
      int occ = 0;
      CC1D_TRY(occupancy(pl.k, pl.max_smem, dev, &occ));
      pl.n_blk = static_cast<int>(cdiv(D, pl.k.d_tile));
      pl.n_tt = static_cast<int>(cdiv(T, pl.k.t_tile));
      const int64_t M = B * pl.n_tt;
      const int64_t cap = static_cast<int64_t>(di.sms) * occ;
      const int64_t pmax = std::max<int64_t>(1, ws_tma / ((W + 1) * D * 4));
      pl.P = static_cast<int>(std::max<int64_t>(1, std::min({M, cap / pl.n_blk, pmax})));
      pl.grid = static_cast<int64_t>(pl.P) * pl.n_blk;
    }
    int occ = 0;
    CC1D_TRY(occupancy(pl.k, pl.max_smem, dev, &occ));
    GenericParams g{};
    g.x = x, g.weight = weight, g.bias = bias, g.init = initial_states, g.seq = seq_idx;
    g.dy = dout, g.dfinal = dfinal_states, g.dx = dx, g.dinit = dinit, g.partials = partials, g.status = di.status;
    g.sxb = stride_x_batch, g.sxt = stride_x_time, g.syb = stride_dout_batch, g.syt = stride_dout_time;
    g.B = static_cast<int>(B), g.T = static_cast<int>(T), g.D = static_cast<int>(D), g.W = static_cast<int>(W);
    g.n_tt = pl.n_tt, g.n_dc = pl.n_blk;
    g.w_dtype = weight_dtype, g.b_dtype = bias_dtype, g.init_dtype = init_dtype, g.silu = silu != 0;
    void* args[] = {&g};
    CC1D_TRY_CUDA(
        cudaLaunchKernel(pl.k.fn, dim3(static_cast<unsigned>(pl.grid)), dim3(pl.k.threads), args, pl.k.smem, stream));
  }

  // Second stage: fixed-order sum over the P partial rows (one warp per column group).
  const int64_t N = (W + 1) * D;
  const bool vec4 = N % 4 == 0 && reinterpret_cast<uintptr_t>(partials) % 16 == 0;
  const int64_t groups = vec4 ? N / 4 : N;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(cdiv(groups, kReduceWarps), 65535)));
  const int rthreads = kReduceWarps * 32;
  if (vec4)
    cc1d_reduce_partials_kernel<4><<<blocks, rthreads, 0, stream>>>(partials, pl.P, static_cast<int>(D),
                                                                    static_cast<int>(W), dweight, weight_dtype,
                                                                    bias ? dbias : nullptr, bias_dtype, grad_f32,
                                                                    bias != nullptr);
  else
    cc1d_reduce_partials_kernel<1><<<blocks, rthreads, 0, stream>>>(partials, pl.P, static_cast<int>(D),
                                                                    static_cast<int>(W), dweight, weight_dtype,
                                                                    bias ? dbias : nullptr, bias_dtype, grad_f32,
                                                                    bias != nullptr);
  CC1D_TRY_CUDA(cudaGetLastError());
  return CC1D_OK;
}


}  // namespace
}  // namespace cc1d

using namespace cc1d;

extern "C" {

int cc1d_abi_version(void) { return 2; }

const char* cc1d_error_string(int code) {
  switch (code) {
    case CC1D_OK: return "success";
    case CC1D_ERR_INVALID: return "invalid argument (size, stride, dtype code or missing pointer)";
    case CC1D_ERR_UNSUPPORTED: return "unsupported width (the largest supported width is 256)";
    case CC1D_ERR_WORKSPACE: return "workspace smaller than cc1d_bwd_workspace_bytes()";
    case CC1D_ERR_CUDA: return "CUDA call failed (see cc1d_last_cuda_error())";
    case CC1D_ERR_SCRATCH_LIMIT:
      return "backward needs more scratch than cc1d_bwd_noalloc's fixed 8 MiB buffer; call cc1d_bwd with a workspace";
    case CC1D_ERR_LAYOUT:
      return "cc1d_bwd_split: dout pieces or dx strides outside the TMA path; concatenate dout and call cc1d_bwd";
    default: return "unknown error";
  }
}

int cc1d_last_cuda_error(void) { return t_last_cuda_error; }

int cc1d_selftest_wait_timeout(void* stream_) {
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  cc1d_wait_timeout_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream_)>>>(di.status);
  CC1D_TRY_CUDA(cudaGetLastError());
  return CC1D_OK;
}

int cc1d_status(uint32_t* status, int clear) {
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  CC1D_TRY_CUDA(cudaDeviceSynchronize());
  unsigned v = 0;
  CC1D_TRY_CUDA(cudaMemcpy(&v, di.status, sizeof(v), cudaMemcpyDeviceToHost));
  if (clear) CC1D_TRY_CUDA(cudaMemset(di.status, 0, sizeof(unsigned)));
  if (status) *status = v;
  return CC1D_OK;
}

int cc1d_fwd(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight, const void* bias,
             const void* initial_states, const int32_t* seq_idx, void* out, void* final_states, int64_t batch,
             int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int weight_dtype, int bias_dtype,
             int init_dtype, int silu, void* stream_) {
  if (!valid_dtype(x_dtype) || !valid_dtype(weight_dtype) || (bias && !valid_dtype(bias_dtype)) ||
      (initial_states && !valid_dtype(init_dtype)))
    return CC1D_ERR_INVALID;
  CC1D_TRY(check_sizes(batch, seqlen, dim, width));
  if (batch == 0 || dim == 0) return CC1D_OK;
  const int64_t B = batch, T = seqlen, D = dim, W = width, PAD = W - 1;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  if (T == 0) {  // final_states = initial_states, or zero
    if (final_states) CC1D_TRY(launch_fill(final_states, x_dtype, initial_states, init_dtype, B * PAD * D, di.sms, stream));
    return CC1D_OK;
  }
  if (!x || !weight || !out) return CC1D_ERR_INVALID;

  const int es = elem_size(x_dtype);
  const int wt = tma_width(W);
  // The tile kernel runs with TMA loads when x's layout allows, else with plain loads (its output
  // vector stores need rows of a multiple of 8 bytes); other shapes take the generic kernel.
  const bool tma_ok = tma_layout_ok(x, stride_x_batch, stride_x_time, B, D, es);
  if (wt > 0 && (tma_ok || (D * es) % 8 == 0)) {
    const KernelInfo k = fwd_tma_for(x_dtype, wt, seq_idx != nullptr, silu != 0, !tma_ok);
    FwdParams p{};
    if (!tma_ok || encode_3d(&p.tmap_x, x, x_dtype, B, T, D, stride_x_batch, stride_x_time, k.d_tile,
                             k.t_tile + wt - 1)) {
      int occ = 0;
      CC1D_TRY(occupancy(k, k.smem, dev, &occ));  // also raises the kernel's dynamic shared memory limit
      p.x = x, p.weight = weight, p.bias = bias, p.init = initial_states, p.seq = seq_idx;
      p.out = out, p.final_states = final_states, p.status = di.status;
      p.sxb = stride_x_batch, p.sxt = stride_x_time;
      p.B = static_cast<int>(B), p.T = static_cast<int>(T), p.D = static_cast<int>(D), p.W = static_cast<int>(W);
      p.n_tt = static_cast<int>(cdiv(T, k.t_tile));
      p.n_db = static_cast<int>(cdiv(D, k.d_tile));
      p.w_dtype = weight_dtype, p.b_dtype = bias_dtype, p.init_dtype = init_dtype;
      // One CTA per (channel block, time tile, batch row): a 3-D grid when the time tiles and batch
      // rows fit its y and z limits (no index arithmetic in the kernel), else a flat one.
      const int64_t grid = B * p.n_tt * p.n_db;
      if (grid >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
      const dim3 g3 = (p.n_tt <= 65535 && B <= 65535)
                          ? dim3(static_cast<unsigned>(p.n_db), static_cast<unsigned>(p.n_tt), static_cast<unsigned>(B))
                          : dim3(static_cast<unsigned>(grid));
      void* args[] = {&p};
      CC1D_TRY_CUDA(cudaLaunchKernel(k.fn, g3, dim3(k.threads), args, k.smem, stream));
      return CC1D_OK;
    }
  }
  // Generic path.
  const KernelInfo k = fwd_generic_for(x_dtype, static_cast<int>(W));
  int occ = 0;
  CC1D_TRY(occupancy(k, generic_fwd_smem(kGenericMaxWidth), dev, &occ));
  GenericParams g{};
  g.x = x, g.weight = weight, g.bias = bias, g.init = initial_states, g.seq = seq_idx;
  g.out = out, g.final_states = final_states, g.status = di.status;
  g.sxb = stride_x_batch, g.sxt = stride_x_time;
  g.B = static_cast<int>(B), g.T = static_cast<int>(T), g.D = static_cast<int>(D), g.W = static_cast<int>(W);
  g.n_tt = static_cast<int>(cdiv(T, GT));
  g.n_dc = static_cast<int>(cdiv(D, GC));
  g.w_dtype = weight_dtype, g.b_dtype = bias_dtype, g.init_dtype = init_dtype, g.silu = silu != 0;
  const int64_t grid = B * g.n_tt * g.n_dc;
  if (grid >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
  void* args[] = {&g};
  CC1D_TRY_CUDA(cudaLaunchKernel(k.fn, dim3(static_cast<unsigned>(grid)), dim3(k.threads), args, k.smem, stream));
  return CC1D_OK;
}

int cc1d_seq_idx_from_cu_seqlens(const int32_t* cu_seqlens, int64_t n_seqs, int32_t* seq_idx, int64_t batch,
                                 int64_t seqlen, void* stream_) {
  if (n_seqs < 1 || batch < 0 || seqlen < 0 || batch >= (int64_t(1) << 31) || seqlen >= (int64_t(1) << 31) ||
      n_seqs >= (int64_t(1) << 31))
    return CC1D_ERR_INVALID;
  if (batch == 0 || seqlen == 0) return CC1D_OK;
  if (!cu_seqlens || !seq_idx) return CC1D_ERR_INVALID;
  const int64_t n = batch * seqlen;
  if (cdiv(n, 256) >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
  cc1d_seq_idx_kernel<<<static_cast<unsigned>(cdiv(n, 256)), 256, 0, static_cast<cudaStream_t>(stream_)>>>(
      cu_seqlens, static_cast<int>(n_seqs), seq_idx, static_cast<int>(batch), static_cast<int>(seqlen));
  CC1D_TRY_CUDA(cudaGetLastError());
  return CC1D_OK;
}

int cc1d_update(const void* x, int64_t stride_x_batch, int64_t stride_x_time, void* conv_state,
                const int32_t* state_indices, const void* weight, const void* bias, void* out, int64_t batch,
                int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int state_dtype, int weight_dtype,
                int bias_dtype, int silu, void* stream_) {
  if (!valid_dtype(x_dtype) || !valid_dtype(state_dtype) || !valid_dtype(weight_dtype) ||
      (bias && !valid_dtype(bias_dtype)))
    return CC1D_ERR_INVALID;
  CC1D_TRY(check_sizes(batch, seqlen, dim, width));
  if (batch == 0 || dim == 0 || seqlen == 0) return CC1D_OK;
  if (!x || !conv_state || !weight || !out) return CC1D_ERR_INVALID;
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  UpdateParams u{};
  u.x = x, u.state = conv_state, u.indices = state_indices, u.weight = weight, u.bias = bias, u.out = out;
  u.sxb = stride_x_batch, u.sxt = stride_x_time;
  u.B = static_cast<int>(batch), u.L = static_cast<int>(seqlen), u.D = static_cast<int>(dim), u.W = static_cast<int>(width);
  u.x_dtype = x_dtype, u.s_dtype = state_dtype, u.w_dtype = weight_dtype, u.b_dtype = bias_dtype, u.silu = silu != 0;
  const int64_t n = batch * dim;
  if (cdiv(n, 256) >= (int64_t(1) << 31)) return CC1D_ERR_INVALID;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const void* kernel = update_vec_kernel(x_dtype, state_dtype, static_cast<int>(width));
  const int64_t cpt = x_dtype == kF32 ? 2 : 4;  // channels of one 8-byte vector
  const bool vec = kernel != nullptr && dim % cpt == 0 && reinterpret_cast<uintptr_t>(x) % 8 == 0 &&
                   reinterpret_cast<uintptr_t>(conv_state) % 8 == 0 && reinterpret_cast<uintptr_t>(out) % 8 == 0 &&
                   stride_x_batch % cpt == 0 && stride_x_time % cpt == 0;
  if (vec) {
    void* args[] = {&u};
    CC1D_TRY_CUDA(cudaLaunchKernel(kernel, dim3(static_cast<unsigned>(cdiv(n / cpt, 256))), dim3(256), args, 0, stream));
  } else {
    cc1d_update_kernel<<<static_cast<unsigned>(cdiv(n, 256)), 256, 0, stream>>>(u);
    CC1D_TRY_CUDA(cudaGetLastError());
  }
  return CC1D_OK;
}

int cc1d_copy_channels(void* dst, int64_t dst_stride_batch, int64_t dst_stride_time, const void* src,
                       int64_t src_stride_batch, int64_t src_stride_time, int64_t batch, int64_t seqlen,
                       int64_t channels, int elem_bytes, void* stream_) {
  if (batch < 0 || seqlen < 0 || channels < 0 || (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 &&
                                                  elem_bytes != 8))
    return CC1D_ERR_INVALID;
  if (batch == 0 || seqlen == 0 || channels == 0) return CC1D_OK;
  if (!dst || !src) return CC1D_ERR_INVALID;
  CopyParams c{};
  c.src = static_cast<const unsigned char*>(src), c.dst = static_cast<unsigned char*>(dst);
  c.src_sb = src_stride_batch * elem_bytes, c.src_st = src_stride_time * elem_bytes;
  c.dst_sb = dst_stride_batch * elem_bytes, c.dst_st = dst_stride_time * elem_bytes;
  c.T = seqlen, c.rows = batch * seqlen;
  const int64_t row_bytes = channels * elem_bytes;
  uint64_t g = static_cast<uint64_t>(row_bytes) | reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) |
               static_cast<uint64_t>(c.src_st) | static_cast<uint64_t>(c.dst_st);
  if (batch > 1) g |= static_cast<uint64_t>(c.src_sb) | static_cast<uint64_t>(c.dst_sb);
  const int vb = g % 16 == 0 ? 16 : g % 8 == 0 ? 8 : g % 4 == 0 ? 4 : g % 2 == 0 ? 2 : 0;
  if (vb == 0) return CC1D_ERR_INVALID;  // single bytes: not a channel block of this library's types
  c.vpr = row_bytes / vb;
  DeviceInfo di;
  int dev = 0;
  CC1D_TRY(device_info(&di, &dev));
  const int64_t n = c.rows * c.vpr;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(cdiv(n, 256), int64_t(di.sms) * 16));
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  switch (vb) {
    case 16: cc1d_copy_channels_kernel<16><<<blocks, 256, 0, stream>>>(c); break;
    case 8: cc1d_copy_channels_kernel<8><<<blocks, 256, 0, stream>>>(c); break;
    case 4: cc1d_copy_channels_kernel<4><<<blocks, 256, 0, stream>>>(c); break;
    default: cc1d_copy_channels_kernel<2><<<blocks, 256, 0, stream>>>(c); break;
  }
  CC1D_TRY_CUDA(cudaGetLastError());
  return CC1D_OK;
}

int64_t cc1d_bwd_workspace_bytes(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* dout,
                                 int64_t stride_dout_batch, int64_t stride_dout_time, int64_t batch, int64_t seqlen,
                                 int64_t dim, int64_t width, int x_dtype) {
  int64_t bytes = 0;
  if (workspace_need(x, stride_x_batch, stride_x_time, dout, stride_dout_batch, stride_dout_time, batch, seqlen, dim,
                     width, x_dtype, &bytes) != CC1D_OK)
    return -1;
  return bytes;
}

int cc1d_bwd(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight, const void* bias,
             const void* initial_states, const int32_t* seq_idx, const void* dout, int64_t stride_dout_batch,
             int64_t stride_dout_time, const void* dfinal_states, void* dx, void* dweight, void* dbias, void* dinit,
             float* grad_f32, void* workspace, int64_t workspace_bytes, int64_t batch, int64_t seqlen, int64_t dim,
             int64_t width, int x_dtype, int weight_dtype, int bias_dtype, int init_dtype, int silu, void* stream_) {
  const cc1d_dout_piece piece{dout, stride_dout_batch, stride_dout_time, dim};
  return bwd_impl(x, stride_x_batch, stride_x_time, weight, bias, initial_states, seq_idx, &piece, 1, dfinal_states, dx,
                  seqlen * dim, dim, dweight, dbias, dinit, grad_f32, workspace, workspace_bytes, batch, seqlen, dim,
                  width, x_dtype, weight_dtype, bias_dtype, init_dtype, silu, stream_, false);
}

int cc1d_bwd_split(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight,
                   const void* bias, const void* initial_states, const int32_t* seq_idx,
                   const cc1d_dout_piece* dout_pieces, int n_pieces, const void* dfinal_states, void* dx,
                   int64_t stride_dx_batch, int64_t stride_dx_time, void* dweight, void* dbias, void* dinit,
                   float* grad_f32, void* workspace, int64_t workspace_bytes, int64_t batch, int64_t seqlen,
                   int64_t dim, int64_t width, int x_dtype, int weight_dtype, int bias_dtype, int init_dtype,
                   int silu, void* stream_) {
  if (dout_pieces == nullptr || n_pieces < 1 || n_pieces > kMaxDoutPieces) return CC1D_ERR_INVALID;
  int64_t sum = 0;
  for (int i = 0; i < n_pieces; ++i) {
    if (dout_pieces[i].channels <= 0) return CC1D_ERR_INVALID;
    sum += dout_pieces[i].channels;
  }
  if (sum != dim) return CC1D_ERR_INVALID;
  return bwd_impl(x, stride_x_batch, stride_x_time, weight, bias, initial_states, seq_idx, dout_pieces, n_pieces,
                  dfinal_states, dx, stride_dx_batch, stride_dx_time, dweight, dbias, dinit, grad_f32, workspace,
                  workspace_bytes, batch, seqlen, dim, width, x_dtype, weight_dtype, bias_dtype, init_dtype, silu,
                  stream_, true);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// cc1d_bwd_noalloc: the backward for callers that cannot allocate device memory.
//
// cc1d_bwd needs a caller-provided device workspace for its per-CTA weight/bias partial sums.
// Some callers have no way to provide one: an inference or training runtime that carves all of
// device memory into its own arena at start-up and must not call cudaMalloc afterwards (the call
// can fail or fragment the arena), a latency-critical path where cudaMalloc/cudaFree may
// synchronise the whole device, or host code that reaches this library only through its C ABI
// (an FFI binding) with no device allocator of its own. For them the partial sums live in a
// fixed array in the library's own device memory instead, sized for ordinary shapes.
//
// Limits and behaviour:
//  - The array holds kNoAllocScratchBytes (8 MiB). A call whose plan needs more (the same number
//    cc1d_bwd_workspace_bytes returns) is rejected with CC1D_ERR_SCRATCH_LIMIT before any device
//    work; use cc1d_bwd with a workspace for it.
//  - The array exists once per GPU that loads the library, and stays allocated until the process
//    exits.
//  - Nothing is allocated here: no cudaMalloc, cudaFree or allocating library routine. The
//    kernels write every partial they later read, so no part of the array has to start at zero
//    and nothing is cleared between calls; the array keeps the last call's partial sums.
//  - Every call on a device shares the one array, so calls that overlap on the GPU (different
//    streams, no ordering between them) race on it and give wrong gradients. Order them (one
//    stream, or events).
//  - The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress, with that device current; make that first call before any stream
//    capture begins. The address is kept for the life of the process, so cudaDeviceReset on a
//    device after its first call is not supported (the module reloads and the array may move).
//  - Errors are cc1d_bwd's: the same sizes, dtypes and device give the same code.
// ---------------------------------------------------------------------------------------------
namespace cc1d {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once per device.
int noalloc_scratch(void** out) {
  int dev = 0;
  CC1D_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return CC1D_ERR_INVALID;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    CC1D_TRY_CUDA(cudaGetSymbolAddress(&ptr, g_noalloc_scratch));
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return CC1D_OK;
}

}  // namespace
}  // namespace cc1d

extern "C" int cc1d_bwd_noalloc(const void* x, int64_t stride_x_batch, int64_t stride_x_time, const void* weight,
                                const void* bias, const void* initial_states, const int32_t* seq_idx, const void* dout,
                                int64_t stride_dout_batch, int64_t stride_dout_time, const void* dfinal_states,
                                void* dx, void* dweight, void* dbias, void* dinit, float* grad_f32, int64_t batch,
                                int64_t seqlen, int64_t dim, int64_t width, int x_dtype, int weight_dtype,
                                int bias_dtype, int init_dtype, int silu, void* stream) {
  int64_t need = 0;
  const int prc = cc1d::workspace_need(x, stride_x_batch, stride_x_time, dout, stride_dout_batch, stride_dout_time,
                                       batch, seqlen, dim, width, x_dtype, &need);
  if (prc != CC1D_OK) return prc;
  if (static_cast<uint64_t>(need) > cc1d::kNoAllocScratchBytes) return CC1D_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int rc = cc1d::noalloc_scratch(&scratch);
  if (rc != CC1D_OK) return rc;
  return cc1d_bwd(x, stride_x_batch, stride_x_time, weight, bias, initial_states, seq_idx, dout, stride_dout_batch,
                  stride_dout_time, dfinal_states, dx, dweight, dbias, dinit, grad_f32, scratch,
                  static_cast<int64_t>(cc1d::kNoAllocScratchBytes), batch, seqlen, dim, width, x_dtype, weight_dtype,
                  bias_dtype, init_dtype, silu, stream);
}
