// capi.cu -- the extern "C" boundary declared in include/cobra_b200.h.
//
// Validates shapes and pointers, carves the caller's workspace, builds the TMA
// tensor maps (cuTensorMapEncodeTiled through the runtime's driver entry
// point, so no libcuda link is needed) and launches the kernels on the
// caller's stream. Nothing here allocates, synchronises (except
// b200l_read_status, which exists to do so) or keeps state other than a
// per-device cache of kernel attributes and device properties.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_set>

#include "../../include/cobra_b200.h"
#include "attn.cuh"
#include "attn2.cuh"
#include "common.cuh"
#include "fused_layer.cuh"
#include "gemm.cuh"
#include "rowln.cuh"

using namespace b200l;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(B200L_ERR_LAUNCH, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// ---------------------------------------------------------------- device cache
struct DevInfo {
  int sms = 0;
  int major = 0;
  bool ok = false;
};
std::mutex g_mu;
DevInfo g_dev[64];
std::unordered_set<unsigned long long> g_attr_done;

int device_info(DevInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B200L_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev[dev].ok) {
    int sms = 0, major = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(SM count)");
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute(cc major)");
    g_dev[dev].sms = sms;
    g_dev[dev].major = major;
    g_dev[dev].ok = true;
  }
  *out = g_dev[dev];
  if (out->major != 10) return fail(B200L_ERR_DEVICE, "device %d has compute capability %d.x, need 10.x (sm_100a)", dev, out->major);
  return B200L_OK;
}

// Sets the dynamic shared memory limit of a kernel once per device.
int ensure_smem(const void* func, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  const unsigned long long key = reinterpret_cast<unsigned long long>(func) * 131ull + (unsigned long long)dev;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_attr_done.count(key)) return B200L_OK;
  }
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(MaxDynamicSharedMemorySize)");
  std::lock_guard<std::mutex> lk(g_mu);
  g_attr_done.insert(key);
  return B200L_OK;
}

// ---------------------------------------------------------------- tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// fp16 tensor of rank 2 or 3; dims/strides innermost first, strides in bytes
// for dims 1.. ; box innermost first.
int make_map(CUtensorMap* map, const void* base, int rank, const unsigned long long* dims,
             const unsigned long long* strides_bytes, const unsigned* box, CUtensorMapSwizzle swz, const char* what,
             CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(B200L_ERR_LAUNCH, "cuTensorMapEncodeTiled unavailable from the driver");
  cuuint64_t gd[3], gs[2];
  cuuint32_t bx[3], es[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
  }
  for (int i = 0; i + 1 < rank; ++i) gs[i] = strides_bytes[i];
  CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(B200L_ERR_LAUNCH, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", what, (int)r);
  return B200L_OK;
}

int map_rows_k(CUtensorMap* map, const void* base, unsigned long long rows, int k, unsigned box_rows,
               const char* what) {
  const unsigned long long dims[2] = {(unsigned long long)k, rows};
  const unsigned long long strides[1] = {(unsigned long long)k * 2};
  const unsigned box[2] = {64, box_rows};
  return make_map(map, base, 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, what);
}

// ---------------------------------------------------------------- plan
size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Plan {
  int B, S, d, H, dh, dhp, sp;
  int Hl, dq;          // heads K1 / K2 compute (local_heads, or all H) and their width Hl * dh
  long long T;
  size_t off_q, off_k, off_vt, off_ctx, off_h;
  size_t total;        // status block + every intermediate: what K1 / K2 / K3 one at a time need
  bool fused;          // b200l_layer_forward runs the whole-layer kernel
  size_t layer_total;  // what b200l_layer_forward needs: the status block alone when fused
};

// Whole-layer kernel for d_model in {64, 128}, head_dim 32, S <= 128.
bool fused_shape(int S, int d, int dh) { return (d == 64 || d == 128) && dh == 32 && S <= 128; }

int make_plan(const b200l_layer_desc* desc, Plan* p) {
  if (!desc) return fail(B200L_ERR_NULL_POINTER, "layer descriptor is NULL");
  const int B = desc->batch, S = desc->seq_len, d = desc->d_model, H = desc->num_heads;
  if (B <= 0 || S <= 0 || d <= 0 || H <= 0)
    return fail(B200L_ERR_BAD_SHAPE, "batch, seq_len, d_model and num_heads must be positive (got %d, %d, %d, %d)", B, S, d, H);
  if (d % H != 0) return fail(B200L_ERR_BAD_SHAPE, "d_model (%d) must be divisible by num_heads (%d)", d, H);
  const int dh = d / H;
  if (dh % 32 != 0 || dh > 256)
    return fail(B200L_ERR_UNSUPPORTED_HEAD_DIM, "head_dim %d unsupported: need a multiple of 32 in [32, 256]", dh);
  if (d > 2048) return fail(B200L_ERR_BAD_SHAPE, "d_model %d > 2048 is not supported", d);
  const long long T = (long long)B * S;
  const int dhp = dh <= 32 ? 32 : dh <= 64 ? 64 : dh <= 128 ? 128 : 256;
  const int sp = (S + 7) / 8 * 8;
  if ((long long)B * H * ((S + 127) / 128) > 0x7fffffffLL || T > 0x7fffffffLL)
    return fail(B200L_ERR_BAD_SHAPE, "problem too large for 32-bit tile indices");
  if (desc->local_heads < 0 || desc->local_heads > H)
    return fail(B200L_ERR_BAD_SHAPE, "local_heads %d must be in [0, num_heads = %d]", desc->local_heads, H);
  const int Hl = desc->local_heads ? desc->local_heads : H;
  p->B = B; p->S = S; p->d = d; p->H = H; p->dh = dh; p->dhp = dhp; p->sp = sp; p->T = T;
  p->Hl = Hl; p->dq = Hl * dh;
  size_t off = 1024;  // status block (256 B) padded to keep every region 1024-aligned
  const size_t qk = (size_t)B * Hl * S * dhp * 2;
  p->off_q = off; off = align_up(off + qk, 1024);
  p->off_k = off; off = align_up(off + qk, 1024);
  p->off_vt = off; off = align_up(off + (size_t)B * Hl * dhp * sp * 2, 1024);
  p->off_ctx = off; off = align_up(off + (size_t)T * p->dq * 2, 1024);
  p->off_h = off;
  if (d > 256) off = align_up(off + (size_t)T * d * 2, 1024);
  p->total = off;
  // The whole-layer kernel keeps h, q, k, v and ctx on chip: it touches only
  // the status block.
  p->fused = fused_shape(S, d, dh) && Hl == H;
  p->layer_total = p->fused ? 1024 : p->total;
  return B200L_OK;
}

// whole_layer: the caller is b200l_layer_forward (workspace sized by the path
// it takes); otherwise a per-kernel entry point (every intermediate).
int check_common(const b200l_layer_desc* desc, const void* ws, size_t ws_bytes, Plan* p, DevInfo* dev,
                 bool whole_layer = false) {
  int rc = make_plan(desc, p);
  if (rc) return rc;
  if ((rc = device_info(dev))) return rc;
  if (!ws) return fail(B200L_ERR_NULL_POINTER, "workspace is NULL");
  if (reinterpret_cast<uintptr_t>(ws) % 1024) return fail(B200L_ERR_ALIGNMENT, "workspace must be 1024-byte aligned");
  const size_t need = whole_layer ? p->layer_total : p->total;
  if (ws_bytes < need)
    return fail(B200L_ERR_WORKSPACE_TOO_SMALL, "workspace has %zu bytes, need %zu%s", ws_bytes, need,
                whole_layer ? "" : " (the per-kernel entry points need b200l_kernel_workspace_bytes)");
  const void* ptrs[] = {desc->wqkv, desc->bqkv, desc->wo, desc->bo, desc->ln1_w, desc->ln1_b, desc->ln2_w, desc->ln2_b};
  const char* names[] = {"wqkv", "bqkv", "wo", "bo", "ln1_w", "ln1_b", "ln2_w", "ln2_b"};
  for (int i = 0; i < 8; ++i) {
    if (!ptrs[i]) return fail(B200L_ERR_NULL_POINTER, "%s is NULL", names[i]);
    if (reinterpret_cast<uintptr_t>(ptrs[i]) % 16) return fail(B200L_ERR_ALIGNMENT, "%s must be 16-byte aligned", names[i]);
  }
  return B200L_OK;
}

QkvOut qkv_out(const Plan& p, void* ws) {
  uint8_t* w = static_cast<uint8_t*>(ws);
  QkvOut o;
  o.q = reinterpret_cast<__half*>(w + p.off_q);
  o.k = reinterpret_cast<__half*>(w + p.off_k);
  o.vt = reinterpret_cast<__half*>(w + p.off_vt);
  o.S = p.S; o.H = p.Hl; o.dh = p.dh; o.dhp = p.dhp; o.sp = p.sp; o.dq = p.dq;
  return o;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, what);
  return B200L_OK;
}

// ---------------------------------------------------------------- launches
// Launch with programmatic stream serialisation: the grid may be scheduled
// while the previous kernel on the stream finishes; every layer kernel starts
// with griddepcontrol.wait (pdl_wait_then_release), so none of its work runs
// before its predecessor has completed.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <int VPL, bool F16>
int launch_row_ln_t(const float* in, void* out, const float* w, const float* b, float eps, long long T, int d,
                    cudaStream_t st, const uint8_t* rowmask) {
  const long long blocks = (T + 7) / 8;
  cudaError_t e = launch_pdl(row_ln_kernel<VPL, F16>, dim3((unsigned)blocks), dim3(256), 0, st, in, out, w, b, eps, T, d,
                             rowmask);
  if (e != cudaSuccess) return cuda_fail(e, "row_ln_kernel");
  return check_launch("row_ln_kernel");
}
template <bool F16>
int launch_row_ln(const float* in, void* out, const float* w, const float* b, float eps, long long T, int d,
                  cudaStream_t st, const uint8_t* rowmask = nullptr) {
  const int v = (d + 127) / 128;
  if (v <= 1) return launch_row_ln_t<1, F16>(in, out, w, b, eps, T, d, st, rowmask);
  if (v <= 2) return launch_row_ln_t<2, F16>(in, out, w, b, eps, T, d, st, rowmask);
  if (v <= 4) return launch_row_ln_t<4, F16>(in, out, w, b, eps, T, d, st, rowmask);
  if (v <= 8) return launch_row_ln_t<8, F16>(in, out, w, b, eps, T, d, st, rowmask);
  return launch_row_ln_t<16, F16>(in, out, w, b, eps, T, d, st, rowmask);
}

template <int KP>
int launch_qkv_lnfused_t(const b200l_layer_desc* desc, const Plan& p, const float* x, void* ws, cudaStream_t st) {
  CUtensorMap map_w;
  int rc = map_rows_k(&map_w, desc->wqkv, 3ull * p.dq, p.d, 128, "wqkv");
  if (rc) return rc;
  auto kern = qkv_lnfused_kernel<KP>;
  const int smem = QkvLnFusedCfg<KP>::SMEM;
  if ((rc = ensure_smem((const void*)kern, smem))) return rc;
  const long long blocks = (p.T + 127) / 128;
  cudaError_t e = launch_pdl(kern, dim3((unsigned)blocks), dim3(256), smem, st, map_w, x, desc->ln1_w, desc->ln1_b,
                             desc->eps1, desc->bqkv, qkv_out(p, ws), p.T, p.d, 3 * p.dq,
                             reinterpret_cast<DevStatus*>(ws));
  if (e != cudaSuccess) return cuda_fail(e, "qkv_lnfused_kernel");
  return check_launch("qkv_lnfused_kernel");
}

template <int BN, int ST, int EPI>
int launch_gemm_tma_t(const CUtensorMap& map_a, const CUtensorMap& map_b, const EpiArgs& ea, long long T, int K, int N,
                      void* ws, cudaStream_t st, const QkvMaps* qm = nullptr) {
  auto kern = gemm_tma_kernel<BN, ST, EPI>;
  const int smem = EPI == EPI_QKV ? GemmTmaCfg<BN, ST>::SMEM_QKV : GemmTmaCfg<BN, ST>::SMEM;
  QkvMaps maps;
  if (qm) maps = *qm;
  else memset(&maps, 0, sizeof maps);
  int rc = ensure_smem((const void*)kern, smem);
  if (rc) return rc;
  DevInfo dev;
  if ((rc = device_info(&dev))) return rc;
  const long long tiles = ((T + 127) / 128) * ((N + BN - 1) / BN);   // persistent: at most one CTA per SM
  const unsigned grid = (unsigned)(tiles < dev.sms ? tiles : dev.sms);
  cudaError_t e = launch_pdl(kern, dim3(grid), dim3(192), smem, st, map_a, map_b, maps, ea, T, K, N,
                             reinterpret_cast<DevStatus*>(ws));
  if (e != cudaSuccess) return cuda_fail(e, "gemm_tma_kernel");
  return check_launch("gemm_tma_kernel");
}

// Clusters of NC CTAs for the LayerNorm-2 out-projection (d = 256 NC): the
// persistent grid holds as many clusters as can be resident at once (looked
// up once per device and kernel), at most one per M tile.
template <int NC, int ST, int BN = 256>
int launch_gemm_ln_cluster_t(const CUtensorMap& map_a, const CUtensorMap& map_b, const EpiArgs& ea, long long T,
                             int K, void* ws, cudaStream_t st) {
  using Cfg = GemmLnClusterCfg<NC, ST, BN>;
  auto kern = gemm_ln_cluster_kernel<NC, ST, BN>;
  const int smem = Cfg::SMEM;
  int rc = ensure_smem((const void*)kern, smem);
  if (rc) return rc;
  // x and y as [T, d] fp32 in 128B-swizzled boxes of 32 columns: 128 rows for
  // the residual's chunks, one warp's 32 rows for the output's.
  CUtensorMap map_x, map_y;
  {
    const unsigned long long dims[2] = {(unsigned long long)ea.d, (unsigned long long)T};
    const unsigned long long strides[1] = {(unsigned long long)ea.d * 4};
    const unsigned box_x[2] = {32, 128}, box_y[2] = {32, 32};
    if ((rc = make_map(&map_x, ea.x, 2, dims, strides, box_x, CU_TENSOR_MAP_SWIZZLE_128B, "x",
                       CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
    if ((rc = make_map(&map_y, ea.y, 2, dims, strides, box_y, CU_TENSOR_MAP_SWIZZLE_128B, "y",
                       CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = NC;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see launch_pdl
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  static int max_clusters[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B200L_ERR_DEVICE, "device ordinal %d out of range", dev);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (max_clusters[dev] == 0) {
      cfg.gridDim = dim3(NC * 16, 1, 1);
      cfg.numAttrs = 1;   // the occupancy query sees the cluster shape only
      int n = 0;
      e = cudaOccupancyMaxActiveClusters(&n, (const void*)kern, &cfg);
      cfg.numAttrs = 2;
      if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters");
      if (n <= 0) return fail(B200L_ERR_LAUNCH, "no cluster of %d CTAs fits on this device", NC);
      max_clusters[dev] = n;
    }
  }
  const long long MT = (T + 127) / 128;
  const long long ncl = MT < max_clusters[dev] ? MT : max_clusters[dev];
  cfg.gridDim = dim3((unsigned)(ncl * NC), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, map_a, map_b, map_x, map_y, ea, T, K, reinterpret_cast<DevStatus*>(ws));
  if (e != cudaSuccess) return cuda_fail(e, "cudaLaunchKernelEx(gemm_ln_cluster_kernel)");
  return check_launch("gemm_ln_cluster_kernel");
}

int run_qkv(const b200l_layer_desc* desc, const Plan& p, const float* x, void* ws, cudaStream_t st) {
  if (p.d <= 256) {
    const int kp = (p.d + 63) / 64 * 64;
    switch (kp) {
      case 64: return launch_qkv_lnfused_t<64>(desc, p, x, ws, st);
      case 128: return launch_qkv_lnfused_t<128>(desc, p, x, ws, st);
      case 192: return launch_qkv_lnfused_t<192>(desc, p, x, ws, st);
      default: return launch_qkv_lnfused_t<256>(desc, p, x, ws, st);
    }
  }
  // d > 256: row LayerNorm to fp16 h, then the TMA-fed GEMM with the QKV epilogue.
  __half* h = reinterpret_cast<__half*>(static_cast<uint8_t*>(ws) + p.off_h);
  int rc = launch_row_ln<true>(x, h, desc->ln1_w, desc->ln1_b, desc->eps1, p.T, p.d, st);
  if (rc) return rc;
  CUtensorMap map_a, map_b;
  if ((rc = map_rows_k(&map_a, h, (unsigned long long)p.T, p.d, 128, "h"))) return rc;
  if ((rc = map_rows_k(&map_b, desc->wqkv, 3ull * p.dq, p.d, 256, "wqkv"))) return rc;
  EpiArgs ea{};
  ea.qkv = qkv_out(p, ws);
  ea.bias = desc->bqkv;
  ea.d = p.d;
  // q, k [B*Hl, S, dhp] and v^T [B*Hl, dhp, sp] in 32 x 32 boxes (64-byte
  // swizzle) for the epilogue's TMA stores.
  QkvMaps qm;
  memset(&qm, 0, sizeof qm);
  {
    uint8_t* w = static_cast<uint8_t*>(ws);
    const unsigned long long bh = (unsigned long long)p.B * p.Hl;
    const unsigned long long dq[3] = {(unsigned long long)p.dhp, (unsigned long long)p.S, bh};
    const unsigned long long sq[2] = {(unsigned long long)p.dhp * 2, (unsigned long long)p.S * p.dhp * 2};
    const unsigned long long dv[3] = {(unsigned long long)p.sp, (unsigned long long)p.dhp, bh};
    const unsigned long long sv[2] = {(unsigned long long)p.sp * 2, (unsigned long long)p.dhp * p.sp * 2};
    const unsigned box[3] = {32, 32, 1};
    if ((rc = make_map(&qm.q, w + p.off_q, 3, dq, sq, box, CU_TENSOR_MAP_SWIZZLE_64B, "q box"))) return rc;
    if ((rc = make_map(&qm.k, w + p.off_k, 3, dq, sq, box, CU_TENSOR_MAP_SWIZZLE_64B, "k box"))) return rc;
    if ((rc = make_map(&qm.vt, w + p.off_vt, 3, dv, sv, box, CU_TENSOR_MAP_SWIZZLE_64B, "v^T box"))) return rc;
    qm.use = 1;
  }
  // Three stages (144 KB) of the operand ring; with four stages it measured
  // 4 % slower.
  return launch_gemm_tma_t<256, 3, EPI_QKV>(map_a, map_b, ea, p.T, p.d, 3 * p.dq, ws, st, &qm);
}

// TWO_TILE: the two-query-tile kernel with P in TMEM (head_dim <= 64);
// otherwise one query tile per item with P in shared memory.
template <int DHP, int BN, bool TWO_TILE = false>
int launch_attn_t(const b200l_layer_desc* desc, const Plan& p, const DevInfo& dev, void* ws, cudaStream_t st) {
  uint8_t* w = static_cast<uint8_t*>(ws);
  const unsigned long long BH = (unsigned long long)p.B * p.Hl;
  CUtensorMap mq, mk, mv;
  const CUtensorMapSwizzle qk_swz = DHP >= 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const unsigned qk_inner = DHP >= 64 ? 64 : 32;
  {
    const unsigned long long dims[3] = {(unsigned long long)DHP, (unsigned long long)p.S, BH};
    const unsigned long long strides[2] = {(unsigned long long)DHP * 2, (unsigned long long)p.S * DHP * 2};
    const unsigned box_q[3] = {qk_inner, 128, 1};
    const unsigned box_k[3] = {qk_inner, (unsigned)BN, 1};
    int rc = make_map(&mq, w + p.off_q, 3, dims, strides, box_q, qk_swz, "q");
    if (rc) return rc;
    if ((rc = make_map(&mk, w + p.off_k, 3, dims, strides, box_k, qk_swz, "k"))) return rc;
  }
  {
    const unsigned long long dims[3] = {(unsigned long long)p.S, (unsigned long long)DHP, BH};
    const unsigned long long strides[2] = {(unsigned long long)p.sp * 2, (unsigned long long)DHP * p.sp * 2};
    const unsigned box[3] = {64, (unsigned)DHP, 1};
    int rc = make_map(&mv, w + p.off_vt, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "v^T");
    if (rc) return rc;
  }
  AttnArgs a;
  a.ctx = reinterpret_cast<__half*>(w + p.off_ctx);
  a.B = p.B; a.S = p.S; a.H = p.Hl; a.dh = p.dh; a.d = p.dq;   // ctx rows hold the computed heads
  a.causal = desc->causal ? 1 : 0;
  a.scale_log2 = (float)(1.4426950408889634 / sqrt((double)p.dh));
  a.num_items = (int)(BH * (unsigned long long)((p.S + 127) / 128));
  a.kmask = desc->valid_mask;
  if constexpr (TWO_TILE) {
    auto kern = a.kmask ? attn2_kernel<DHP, true> : attn2_kernel<DHP, false>;
    const int smem = Attn2Cfg<DHP>::SMEM;
    int rc = ensure_smem((const void*)kern, smem);
    if (rc) return rc;
    const long long items = (long long)BH * ((p.S + 255) / 256);
    const int grid = items < dev.sms ? (int)items : dev.sms;
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(Attn2Cfg<DHP>::THREADS), smem, st, mq, mk, mv, a,
                               reinterpret_cast<DevStatus*>(ws));
    if (e != cudaSuccess) return cuda_fail(e, "attn2_kernel");
    return check_launch("attn2_kernel");
  } else {
    auto kern = a.kmask ? attn_kernel<DHP, BN, true> : attn_kernel<DHP, BN, false>;
    const int smem = AttnCfg<DHP, BN>::SMEM;
    int rc = ensure_smem((const void*)kern, smem);
    if (rc) return rc;
    const int grid = a.num_items < dev.sms ? a.num_items : dev.sms;
    cudaError_t e = launch_pdl(kern, dim3(grid), dim3(192), smem, st, mq, mk, mv, a, reinterpret_cast<DevStatus*>(ws));
    if (e != cudaSuccess) return cuda_fail(e, "attn_kernel");
    return check_launch("attn_kernel");
  }
}

int run_attn(const b200l_layer_desc* desc, const Plan& p, const DevInfo& dev, void* ws, cudaStream_t st) {
  switch (p.dhp) {
    case 32: return launch_attn_t<32, 128, true>(desc, p, dev, ws, st);
    case 64: return launch_attn_t<64, 128, true>(desc, p, dev, ws, st);
    case 128: return launch_attn_t<128, 128>(desc, p, dev, ws, st);
    default: return launch_attn_t<256, 64>(desc, p, dev, ws, st);
  }
}

int run_outproj(const b200l_layer_desc* desc, const Plan& p, const float* x, float* y, void* ws, cudaStream_t st) {
  uint8_t* w = static_cast<uint8_t*>(ws);
  const __half* ctx = reinterpret_cast<const __half*>(w + p.off_ctx);
  EpiArgs ea{};
  ea.bias = desc->bo;
  ea.x = x;
  ea.y = y;
  ea.ln_w = desc->ln2_w;
  ea.ln_b = desc->ln2_b;
  ea.eps = desc->eps2;
  ea.d = p.d;
  ea.rowmask = desc->valid_mask;
  CUtensorMap map_a, map_b;
  int rc = map_rows_k(&map_a, ctx, (unsigned long long)p.T, p.d, 128, "ctx");
  if (rc) return rc;
  if (p.d <= 256) {
    const int bn = (p.d + 63) / 64 * 64;
    if ((rc = map_rows_k(&map_b, desc->wo, (unsigned long long)p.d, p.d, (unsigned)bn, "wo"))) return rc;
    if (bn == p.d) {
      // d a multiple of 64: the row fits one CTA's accumulator exactly; the
      // LayerNorm-2 kernel with the residual and y moved by TMA (a cluster of
      // one CTA, so no statistics exchange).
      switch (bn) {
        case 64: return launch_gemm_ln_cluster_t<1, 3, 64>(map_a, map_b, ea, p.T, p.d, ws, st);
        case 128: return launch_gemm_ln_cluster_t<1, 3, 128>(map_a, map_b, ea, p.T, p.d, ws, st);
        case 192: return launch_gemm_ln_cluster_t<1, 3, 192>(map_a, map_b, ea, p.T, p.d, ws, st);
        default: return launch_gemm_ln_cluster_t<1, 3, 256>(map_a, map_b, ea, p.T, p.d, ws, st);
      }
    }
    switch (bn) {
      case 64: return launch_gemm_tma_t<64, 2, EPI_RESID_LN>(map_a, map_b, ea, p.T, p.d, p.d, ws, st);
      case 128: return launch_gemm_tma_t<128, 2, EPI_RESID_LN>(map_a, map_b, ea, p.T, p.d, p.d, ws, st);
      case 192: return launch_gemm_tma_t<192, 3, EPI_RESID_LN>(map_a, map_b, ea, p.T, p.d, p.d, ws, st);
      default: return launch_gemm_tma_t<256, 4, EPI_RESID_LN>(map_a, map_b, ea, p.T, p.d, p.d, ws, st);
    }
  }
  if ((rc = map_rows_k(&map_b, desc->wo, (unsigned long long)p.d, p.d, 256, "wo"))) return rc;
  // d = 256 NC: a cluster of NC CTAs shares each row tile and completes LN2 in
  // the epilogue (row statistics exchanged through distributed shared memory).
  switch (p.d) {
    case 512: return launch_gemm_ln_cluster_t<2, 3>(map_a, map_b, ea, p.T, p.d, ws, st);
    case 768: return launch_gemm_ln_cluster_t<3, 3>(map_a, map_b, ea, p.T, p.d, ws, st);
    case 1024: return launch_gemm_ln_cluster_t<4, 3>(map_a, map_b, ea, p.T, p.d, ws, st);
    case 1536: return launch_gemm_ln_cluster_t<6, 3>(map_a, map_b, ea, p.T, p.d, ws, st);
    case 2048: return launch_gemm_ln_cluster_t<8, 3>(map_a, map_b, ea, p.T, p.d, ws, st);
    default: break;
  }
  // Other widths: the residual in the GEMM epilogue, then a row LayerNorm pass.
  if ((rc = launch_gemm_tma_t<256, 4, EPI_RESID>(map_a, map_b, ea, p.T, p.d, p.d, ws, st))) return rc;
  return launch_row_ln<false>(y, y, desc->ln2_w, desc->ln2_b, desc->eps2, p.T, p.d, st, nullptr);
}

template <int DM>
int launch_fused_t(const b200l_layer_desc* desc, const Plan& p, const DevInfo& dev, const float* x, float* y, void* ws,
                   cudaStream_t st) {
  CUtensorMap map_wqkv, map_wo;
  int rc = map_rows_k(&map_wqkv, desc->wqkv, 3ull * DM, DM, 32, "wqkv");
  if (rc) return rc;
  if ((rc = map_rows_k(&map_wo, desc->wo, (unsigned long long)DM, DM, DM, "wo"))) return rc;
  // x and y viewed as [B][S][d] fp32 in 32-row x 32-column boxes (one row
  // warp's rows of one chunk): rows past S read as zero and are clipped on store.
  CUtensorMap map_x, map_y;
  {
    const unsigned long long dims[3] = {(unsigned long long)DM, (unsigned long long)p.S, (unsigned long long)p.B};
    const unsigned long long strides[2] = {(unsigned long long)DM * 4, (unsigned long long)p.S * DM * 4};
    const unsigned box[3] = {32, 32, 1};
    if ((rc = make_map(&map_x, x, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "x",
                       CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
    if ((rc = make_map(&map_y, y, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B, "y",
                       CU_TENSOR_MAP_DATA_TYPE_FLOAT32)))
      return rc;
  }
  FusedArgs a;
  a.x = x; a.y = y;
  a.ln1_w = desc->ln1_w; a.ln1_b = desc->ln1_b; a.eps1 = desc->eps1;
  a.bqkv = desc->bqkv; a.bo = desc->bo;
  a.ln2_w = desc->ln2_w; a.ln2_b = desc->ln2_b; a.eps2 = desc->eps2;
  a.B = p.B; a.S = p.S; a.causal = desc->causal ? 1 : 0;
  a.scale_log2 = (float)(1.4426950408889634 / sqrt(32.0));
  a.mask = desc->valid_mask;
  auto kern = a.mask ? fused_layer_kernel<DM, true> : fused_layer_kernel<DM, false>;
  const int smem = FusedCfg<DM>::SMEM;
  if ((rc = ensure_smem((const void*)kern, smem))) return rc;
  const int npairs = (p.B + 1) / 2;
  const int grid = npairs < dev.sms ? npairs : dev.sms;
  kern<<<grid, 512, smem, st>>>(map_wqkv, map_wo, map_x, map_y, a, reinterpret_cast<DevStatus*>(ws));
  return check_launch("fused_layer_kernel");
}

int run_fused(const b200l_layer_desc* desc, const Plan& p, const DevInfo& dev, const float* x, float* y, void* ws,
              cudaStream_t st) {
  if (p.d == 128) return launch_fused_t<128>(desc, p, dev, x, y, ws, st);
  return launch_fused_t<64>(desc, p, dev, x, y, ws, st);
}

// ------------------------------------------------------------------ full block
// x1 = x + Attn(LN1(x)); x2 = x1 + W2 gelu(W1 LN2(x1) + b1) + b2, padded rows
// of x2 zeroed -- BaselineTransformerBlock.forward (torch_transformer_benchmark.py
// :141-145), computed as the reference's fused path does (:1274-1292): the
// out-projection keeps the fp32 residual x1, a row pass writes LN2(x1) in
// fp16, the FFN-in GEMM applies bias + exact GELU in its epilogue and the
// FFN-out GEMM adds bias and residual and zeroes padded rows in its.
struct BlockPlan {
  Plan p;
  int f;
  size_t off_x1, off_h2, off_h1, total;
};

int make_block_plan(const b200l_block_desc* bd, BlockPlan* bp) {
  if (!bd) return fail(B200L_ERR_NULL_POINTER, "block descriptor is NULL");
  int rc = make_plan(&bd->layer, &bp->p);
  if (rc) return rc;
  const int f = bd->ffn_dim;
  if (f <= 0 || f % 8 != 0 || f > 65536)
    return fail(B200L_ERR_BAD_SHAPE, "ffn_dim %d unsupported: need a positive multiple of 8, at most 65536", f);
  bp->f = f;
  const Plan& p = bp->p;
  size_t off = align_up(p.total, 1024);
  bp->off_x1 = off; off = align_up(off + (size_t)p.T * p.d * 4, 1024);
  bp->off_h2 = off; off = align_up(off + (size_t)p.T * p.d * 2, 1024);
  bp->off_h1 = off; off = align_up(off + (size_t)p.T * f * 2, 1024);
  bp->total = off;
  return B200L_OK;
}

// y = x + acc + bias over a [T, d] output with K-major fp16 operands (A [T, K],
// B [d, K]); rowmask_zero selects the padded-row rule (keep x / zero the row).
int run_resid_gemm(const void* a, int K, const void* bmat, int d, const float* bias, const float* x, float* y,
                   const uint8_t* rowmask, int rowmask_zero, long long T, void* ws, cudaStream_t st) {
  EpiArgs ea{};
  ea.bias = bias;
  ea.x = x;
  ea.y = y;
  ea.d = d;
  ea.rowmask = rowmask;
  ea.rowmask_zero = rowmask_zero;
  CUtensorMap map_a, map_b;
  int rc = map_rows_k(&map_a, a, (unsigned long long)T, K, 128, "gemm A");
  if (rc) return rc;
  const int bn = d <= 256 ? (d + 63) / 64 * 64 : 256;
  if ((rc = map_rows_k(&map_b, bmat, (unsigned long long)d, K, (unsigned)bn, "gemm B"))) return rc;
  switch (bn) {
    case 64: return launch_gemm_tma_t<64, 2, EPI_RESID>(map_a, map_b, ea, T, K, d, ws, st);
    case 128: return launch_gemm_tma_t<128, 2, EPI_RESID>(map_a, map_b, ea, T, K, d, ws, st);
    case 192: return launch_gemm_tma_t<192, 3, EPI_RESID>(map_a, map_b, ea, T, K, d, ws, st);
    default: return launch_gemm_tma_t<256, 4, EPI_RESID>(map_a, map_b, ea, T, K, d, ws, st);
  }
}

int run_block(const b200l_block_desc* bd, const BlockPlan& bp, const DevInfo& dev, const float* x, float* y,
              void* ws, cudaStream_t st) {
  const b200l_layer_desc* desc = &bd->layer;
  const Plan& p = bp.p;
  uint8_t* w = static_cast<uint8_t*>(ws);
  float* x1 = reinterpret_cast<float*>(w + bp.off_x1);
  __half* h2 = reinterpret_cast<__half*>(w + bp.off_h2);
  __half* h1 = reinterpret_cast<__half*>(w + bp.off_h1);
  int rc;
  if ((rc = run_qkv(desc, p, x, ws, st))) return rc;
  if ((rc = run_attn(desc, p, dev, ws, st))) return rc;
  // x1 = x + (valid row ? ctx Wo^T + bo : 0)
  if ((rc = run_resid_gemm(w + p.off_ctx, p.d, desc->wo, p.d, desc->bo, x, x1, desc->valid_mask, 0, p.T, ws, st)))
    return rc;
  if ((rc = launch_row_ln<true>(x1, h2, desc->ln2_w, desc->ln2_b, desc->eps2, p.T, p.d, st))) return rc;
  {  // h1 = fp16(gelu(h2 W1^T + b1))
    EpiArgs ea{};
    ea.bias = bd->b1;
    ea.h = h1;
    ea.ldh = bp.f;
    CUtensorMap map_a, map_b;
    if ((rc = map_rows_k(&map_a, h2, (unsigned long long)p.T, p.d, 128, "LN2 output"))) return rc;
    if ((rc = map_rows_k(&map_b, bd->w1, (unsigned long long)bp.f, p.d, 256, "ffn_in weight"))) return rc;
    if ((rc = launch_gemm_tma_t<256, 4, EPI_GELU>(map_a, map_b, ea, p.T, p.d, bp.f, ws, st))) return rc;
  }
  // y = valid row ? x1 + h1 W2^T + b2 : 0
  return run_resid_gemm(h1, bp.f, bd->w2, p.d, bd->b2, x1, y, desc->valid_mask, 1, p.T, ws, st);
}

int check_xy(const void* x, const void* y, bool need_y) {
  if (!x) return fail(B200L_ERR_NULL_POINTER, "x is NULL");
  if (reinterpret_cast<uintptr_t>(x) % 16) return fail(B200L_ERR_ALIGNMENT, "x must be 16-byte aligned");
  if (need_y) {
    if (!y) return fail(B200L_ERR_NULL_POINTER, "y is NULL");
    if (reinterpret_cast<uintptr_t>(y) % 16) return fail(B200L_ERR_ALIGNMENT, "y must be 16-byte aligned");
    if (x == y) return fail(B200L_ERR_BAD_SHAPE, "x and y must not alias");
  }
  return B200L_OK;
}

}  // namespace

// ===================================================================== C ABI
extern "C" {

int b200l_version(void) { return B200L_ABI_VERSION; }

int b200l_last_error(char* buf, size_t n) {
  if (buf && n) {
    const size_t k = g_last_error.size() < n - 1 ? g_last_error.size() : n - 1;
    memcpy(buf, g_last_error.data(), k);
    buf[k] = 0;
  }
  return (int)g_last_error.size();
}

size_t b200l_layer_workspace_bytes(const b200l_layer_desc* desc) {
  Plan p;
  if (make_plan(desc, &p)) return 0;
  return p.layer_total;
}

size_t b200l_kernel_workspace_bytes(const b200l_layer_desc* desc) {
  Plan p;
  if (make_plan(desc, &p)) return 0;
  return p.total;
}

int b200l_clear_status(void* workspace, void* stream) {
  if (!workspace) return fail(B200L_ERR_NULL_POINTER, "workspace is NULL");
  cudaError_t e = cudaMemsetAsync(workspace, 0, sizeof(DevStatus), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(status)");
  return B200L_OK;
}

int b200l_debug_arm(void* workspace, int32_t site, uint64_t wait_limit_ns, void* stream) {
  if (!workspace) return fail(B200L_ERR_NULL_POINTER, "workspace is NULL");
  if (site < 0 || site > kSiteGemmOperand) return fail(B200L_ERR_BAD_SHAPE, "unknown fault site %d", site);
  if (wait_limit_ns != 0 && wait_limit_ns < 1000000ull)
    return fail(B200L_ERR_BAD_SHAPE, "wait limit %llu ns is below 1 ms", (unsigned long long)wait_limit_ns);
  debug_arm_kernel<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<DevStatus*>(workspace), site,
                                                                    (unsigned long long)wait_limit_ns);
  return check_launch("debug_arm_kernel");
}

int b200l_read_status(const void* workspace, void* stream) {
  if (!workspace) return fail(B200L_ERR_NULL_POINTER, "workspace is NULL");
  DevStatus s;
  cudaError_t e = cudaMemcpyAsync(&s, workspace, sizeof(s), cudaMemcpyDeviceToHost, static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "reading the status block");
  if (s.code) fail(s.code, "device status %d recorded by kernel %d (block %d, site %d)", s.code, s.kernel, s.block, s.where);
  return s.code;
}

int b200l_pack_weights(int32_t d, const float* wq, const float* wk, const float* wv, const float* bq, const float* bk,
                       const float* bv, const float* wo, void* wqkv16, float* bqkv32, void* wo16, void* stream) {
  if (d <= 0) return fail(B200L_ERR_BAD_SHAPE, "d_model must be positive");
  if (!wq || !wk || !wv || !bq || !bk || !bv || !wo || !wqkv16 || !bqkv32 || !wo16)
    return fail(B200L_ERR_NULL_POINTER, "b200l_pack_weights: NULL pointer");
  DevInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  const long long total = 4LL * d * d;
  const int blocks = (int)((total + 255) / 256 < 4096 ? (total + 255) / 256 : 4096);
  pack_weights_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      d, wq, wk, wv, bq, bk, bv, wo, static_cast<__half*>(wqkv16), bqkv32, static_cast<__half*>(wo16));
  return check_launch("pack_weights_kernel");
}

int b200l_qkv_ln_gemm(const b200l_layer_desc* desc, const float* x, void* workspace, size_t ws_bytes, void* stream) {
  Plan p;
  DevInfo dev;
  int rc = check_common(desc, workspace, ws_bytes, &p, &dev);
  if (rc) return rc;
  if ((rc = check_xy(x, nullptr, false))) return rc;
  return run_qkv(desc, p, x, workspace, static_cast<cudaStream_t>(stream));
}

int b200l_flash_attn(const b200l_layer_desc* desc, void* workspace, size_t ws_bytes, void* stream) {
  Plan p;
  DevInfo dev;
  int rc = check_common(desc, workspace, ws_bytes, &p, &dev);
  if (rc) return rc;
  return run_attn(desc, p, dev, workspace, static_cast<cudaStream_t>(stream));
}

int b200l_outproj_res_ln(const b200l_layer_desc* desc, const float* x, float* y, void* workspace, size_t ws_bytes,
                         void* stream) {
  Plan p;
  DevInfo dev;
  int rc = check_common(desc, workspace, ws_bytes, &p, &dev);
  if (rc) return rc;
  if (p.Hl != p.H) return fail(B200L_ERR_BAD_SHAPE, "the out-projection needs every head's ctx: local_heads must be 0");
  if ((rc = check_xy(x, y, true))) return rc;
  return run_outproj(desc, p, x, y, workspace, static_cast<cudaStream_t>(stream));
}

int b200l_layer_forward(const b200l_layer_desc* desc, const float* x, float* y, void* workspace, size_t ws_bytes,
                        void* stream) {
  Plan p;
  DevInfo dev;
  int rc = check_common(desc, workspace, ws_bytes, &p, &dev, /*whole_layer=*/true);
  if (rc) return rc;
  if (p.Hl != p.H) return fail(B200L_ERR_BAD_SHAPE, "b200l_layer_forward computes every head: local_heads must be 0");
  if ((rc = check_xy(x, y, true))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.fused) return run_fused(desc, p, dev, x, y, workspace, st);
  if ((rc = run_qkv(desc, p, x, workspace, st))) return rc;
  if ((rc = run_attn(desc, p, dev, workspace, st))) return rc;
  return run_outproj(desc, p, x, y, workspace, st);
}

size_t b200l_block_workspace_bytes(const b200l_block_desc* desc) {
  BlockPlan bp;
  if (make_block_plan(desc, &bp)) return 0;
  return bp.total;
}

int b200l_block_forward(const b200l_block_desc* desc, const float* x, float* y, void* workspace, size_t ws_bytes,
                        void* stream) {
  BlockPlan bp;
  int rc = make_block_plan(desc, &bp);
  if (rc) return rc;
  if (bp.p.Hl != bp.p.H) return fail(B200L_ERR_BAD_SHAPE, "b200l_block_forward computes every head: local_heads must be 0");
  if (!desc->w1 || !desc->b1 || !desc->w2 || !desc->b2) return fail(B200L_ERR_NULL_POINTER, "FFN weight is NULL");
  Plan p;
  DevInfo dev;
  if ((rc = check_common(&desc->layer, workspace, ws_bytes, &p, &dev))) return rc;
  if (ws_bytes < bp.total)
    return fail(B200L_ERR_WORKSPACE_TOO_SMALL, "workspace %zu bytes < %zu needed", ws_bytes, bp.total);
  if ((rc = check_xy(x, y, true))) return rc;
  return run_block(desc, bp, dev, x, y, workspace, static_cast<cudaStream_t>(stream));
}

int b200l_row_layernorm(const float* x, float* y, const float* w, const float* b, float eps, int64_t rows,
                        int32_t d, const uint8_t* row_mask, void* stream) {
  if (!x || !y || !w || !b) return fail(B200L_ERR_NULL_POINTER, "row_layernorm: NULL pointer");
  if (rows <= 0 || d <= 0 || d % 4 != 0 || d > 2048)
    return fail(B200L_ERR_BAD_SHAPE, "row_layernorm: rows %lld, d %d (need d a multiple of 4 in [4, 2048])",
                (long long)rows, d);
  if (reinterpret_cast<uintptr_t>(x) % 16 || reinterpret_cast<uintptr_t>(y) % 16)
    return fail(B200L_ERR_ALIGNMENT, "row_layernorm: x and y must be 16-byte aligned");
  DevInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  return launch_row_ln<false>(x, y, w, b, eps, rows, d, static_cast<cudaStream_t>(stream), row_mask);
}

int b200l_convert(const void* src, int32_t src_type, void* dst, int32_t dst_type, int64_t n, void* stream) {
  if (!src || !dst) return fail(B200L_ERR_NULL_POINTER, "convert: NULL pointer");
  if (n <= 0) return fail(B200L_ERR_BAD_SHAPE, "convert: n must be positive");
  if (src_type < 0 || src_type > 2 || dst_type < 0 || dst_type > 2)
    return fail(B200L_ERR_BAD_SHAPE, "convert: element types must be B200L_DTYPE_F32 / _F16 / _BF16");
  if (reinterpret_cast<uintptr_t>(src) % 16 || reinterpret_cast<uintptr_t>(dst) % 16)
    return fail(B200L_ERR_ALIGNMENT, "convert: src and dst must be 16-byte aligned");
  if (src_type == dst_type) return fail(B200L_ERR_BAD_SHAPE, "convert: source and destination types are the same");
  DevInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  const long long vecs = (n + 7) / 8;
  const int blocks = (int)((vecs + 255) / 256 < 8L * dev.sms ? (vecs + 255) / 256 : 8L * dev.sms);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto go = [&](auto kern) {
    kern<<<blocks, 256, 0, st>>>(src, dst, (long long)n);
    return check_launch("convert_kernel");
  };
  if (src_type == kF32 && dst_type == kF16) return go(convert_kernel<kF32, kF16>);
  if (src_type == kF32) return go(convert_kernel<kF32, kBF16>);
  if (src_type == kF16 && dst_type == kF32) return go(convert_kernel<kF16, kF32>);
  if (src_type == kF16) return go(convert_kernel<kF16, kBF16>);
  if (dst_type == kF32) return go(convert_kernel<kBF16, kF32>);
  return go(convert_kernel<kBF16, kF16>);
}

int b200l_cast_f16(const float* src, void* dst, int64_t n, void* stream) {
  if (!src || !dst) return fail(B200L_ERR_NULL_POINTER, "cast_f16: NULL pointer");
  if (n <= 0) return fail(B200L_ERR_BAD_SHAPE, "cast_f16: n must be positive");
  DevInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  const long long blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  cast_f16_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(src, static_cast<__half*>(dst), n);
  return check_launch("cast_f16_kernel");
}

}  // extern "C"

// ===================================================================== no-alloc variant
// b200l_layer_forward_noalloc: the same kernels as b200l_layer_forward (the
// whole-layer kernel where it applies, else K1 -> K2 -> K3), but the scratch
// they need (status block, and for the three-kernel path q, k, v^T, ctx, h)
// lives in a fixed array inside this library instead of a caller-provided
// workspace.
// It exists for callers that cannot call cudaMalloc themselves -- a plugin
// inside a host process whose device memory is owned by its own pool, or a
// latency-critical service that forbids allocation after start-up because
// cudaMalloc/cudaFree synchronise the device.
//
// The array is B200L_NOALLOC_MAX_SCRATCH_BYTES (64 MiB) plus 1 KiB so the
// regions can start on a 1024-byte boundary; every GPU that loads this
// library holds it until the process exits. Device code could name it
// directly, but in host code its name is only a host-side stand-in, so the
// device address is looked up with cudaGetSymbolAddress on the first call on
// each device (with that device current) and cached for the life of the
// process: after a cudaDeviceReset the module may be loaded at another
// address, so a process that resets a device must not call this entry point
// on it again. Device-side failures land in the status block at the start of
// the array; b200l_noalloc_read_status reads it (the next no-alloc call on the
// device clears it).
static __device__ __align__(256) unsigned char g_noalloc_scratch[B200L_NOALLOC_MAX_SCRATCH_BYTES + 1024];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_base[64] = {nullptr};

int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(B200L_ERR_DEVICE, "device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_base[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_base[dev] = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
  }
  *out = g_noalloc_base[dev];
  return B200L_OK;
}
}  // namespace

extern "C" int b200l_layer_forward_noalloc(const b200l_layer_desc* desc, const float* x, float* y, void* stream) {
  Plan p;
  int rc = make_plan(desc, &p);
  if (rc) return rc;
  if (p.layer_total > (size_t)B200L_NOALLOC_MAX_SCRATCH_BYTES)
    return fail(B200L_ERR_WORKSPACE_TOO_SMALL,
                "b200l_layer_forward_noalloc: this problem needs %zu bytes of scratch but the built-in scratch holds "
                "%zu; call b200l_layer_forward with a workspace instead",
                p.layer_total, (size_t)B200L_NOALLOC_MAX_SCRATCH_BYTES);
  void* ws = nullptr;
  if ((rc = noalloc_scratch(&ws))) return rc;
  // The status block must start at zero for this call; everything else the
  // kernels read is written earlier in the same call.
  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(DevStatus), static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(no-alloc status)");
  return b200l_layer_forward(desc, x, y, ws, (size_t)B200L_NOALLOC_MAX_SCRATCH_BYTES, stream);
}

extern "C" int b200l_noalloc_read_status(void* stream) {
  void* ws = nullptr;
  int rc = noalloc_scratch(&ws);
  if (rc) return rc;
  return b200l_read_status(ws, stream);
}
