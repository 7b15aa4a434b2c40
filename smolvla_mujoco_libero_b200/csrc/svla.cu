// libsvla.so: C-ABI entry points (include/svla.h) over the sm_100a kernels.
//
// Host-side responsibilities: argument validation (status 1 with a message), TMA tensor-map encoding,
// template dispatch, and launch-error reporting (status 2).  Nothing here allocates device memory.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <utility>
#include <mutex>
#include <string>

#include "../../include/svla.h"
#include "attention.cuh"
#include "attention_tc.cuh"
#include "calib.cuh"
#include "gemm.cuh"
#include "misc.cuh"
#include "norm.cuh"
#include "flow.cuh"
#include "process.cuh"
#include "rope.cuh"

namespace svla {

__device__ int g_device_error = 0;

namespace {

thread_local std::string t_last_error;

int32_t fail(int32_t code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int32_t fail(int32_t code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  t_last_error = buf;
  return code;
}

int32_t check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SVLA_OK;
}

// Programmatic dependent launch (see pdl_wait in ptx.cuh): on by default, SVLA_PDL=0 turns it off.
bool pdl_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("SVLA_PDL");
    v = (e != nullptr && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <typename... KArgs, typename... Args>
int32_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       const char* name, unsigned cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_x > 1) {  // CTA pairs: clusters of cluster_x consecutive CTAs along x
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = cluster_x;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
  return check_launch(name);
}

template <typename... KArgs, typename... Args>
int32_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, const char* name,
               Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "%s: %s", name, cudaGetErrorString(e));
  return check_launch(name);
}

int* device_error_ptr() {
  // one device-error word per device; the symbol address is per device
  static int* ptrs[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    ptrs[dev] = static_cast<int*>(p);
  }
  return ptrs[dev];
}

// ---------------------------------------------------------------- TMA descriptors
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
  return fn;
}

// 2D row-major [rows, cols] tensor, box [box_rows, box_cols]; cols is the contiguous dimension.
int32_t make_tmap(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t cols,
                  uint64_t rows, uint64_t ld_elems, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SVLA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return fail(SVLA_ERR_ARG, "TMA base address not 16-byte aligned");
  if ((ld_elems * elem_bytes) % 16 != 0) return fail(SVLA_ERR_ARG, "TMA row stride %llu bytes not a multiple of 16",
                                                    (unsigned long long)(ld_elems * elem_bytes));
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld_elems * elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVLA_ERR_ARG, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return SVLA_OK;
}

// ---------------------------------------------------------------- GEMM dispatch
template <Kind K, int BN, int P, int CG = 1>
constexpr int stages_for() {
  constexpr int a = 128 * 128, b = (BN / CG) * 128, raw = KindTraits<K>::kConvert ? BN * 64 : 0;
  constexpr int stage = P * (a + b + raw);
  constexpr int s = (200 * 1024) / stage;
  return s > 8 ? 8 : (s < 2 ? 2 : s);
}

template <Kind K, int BN, int P, Epi E, int CG = 1>
int32_t launch_gemm_inst(const GemmArgs& args, dim3 grid, cudaStream_t stream) {
  constexpr int ST = stages_for<K, BN, P, CG>();
  using S = GemmSmem<K, BN, P, ST, CG>;
  auto kern = gemm_sm100_kernel<K, BN, P, ST, E, CG>;
  static bool configured[64] = {false};  // the attribute is per function and per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(SVLA_ERR_ARG, "device index %d out of range", dev);
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes);
    if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  return launch_cluster(kern, grid, dim3(gemm_threads<K, P, E>()), S::kBytes, stream, "gemm_sm100_kernel", CG, args);
}

template <Kind K, int BN, int P, int CG>
int32_t dispatch_epi(Epi e, const GemmArgs& args, dim3 grid, cudaStream_t st) {
  if constexpr (CG == 2 && (K == Kind::W8A16 || BN < 128)) {
    return fail(SVLA_ERR_ARG, "CTA pairs take I8 / BF16 operands and 128- or 256-column tiles");
  } else if constexpr (P == 2) {
    if (e == Epi::SiluMul) return launch_gemm_inst<K, BN, 2, Epi::SiluMul, CG>(args, grid, st);
    return fail(SVLA_ERR_ARG, "pair GEMMs support only the SILU_MUL epilogue");
  } else {
    switch (e) {
      case Epi::Bf16: return launch_gemm_inst<K, BN, 1, Epi::Bf16, CG>(args, grid, st);
      case Epi::Rope: return launch_gemm_inst<K, BN, 1, Epi::Rope, CG>(args, grid, st);
      case Epi::Resid: return launch_gemm_inst<K, BN, 1, Epi::Resid, CG>(args, grid, st);
      case Epi::F32: return launch_gemm_inst<K, BN, 1, Epi::F32, CG>(args, grid, st);
      default: break;
    }
    if (e == Epi::GeluQuant) return launch_gemm_inst<K, BN, 1, Epi::GeluQuant, CG>(args, grid, st);
    if constexpr (K == Kind::I8) {
      if (e == Epi::I32) return launch_gemm_inst<K, BN, 1, Epi::I32, CG>(args, grid, st);
    }
    if constexpr (K == Kind::BF16) {
      if (e == Epi::SiluBf16) return launch_gemm_inst<K, BN, 1, Epi::SiluBf16, CG>(args, grid, st);
      if (e == Epi::Euler) return launch_gemm_inst<K, BN, 1, Epi::Euler, CG>(args, grid, st);
    }
    return fail(SVLA_ERR_ARG, "epilogue %d not available for operand kind %d", static_cast<int>(e),
                static_cast<int>(K));
  }
}

template <Kind K, int CG>
int32_t dispatch_bn(int bn, int pair, Epi e, const GemmArgs& args, dim3 grid, cudaStream_t st) {
  if (pair) {
    if (bn == 64) return dispatch_epi<K, 64, 2, CG>(e, args, grid, st);
    if (bn == 128) return dispatch_epi<K, 128, 2, CG>(e, args, grid, st);
    return fail(SVLA_ERR_ARG, "pair GEMMs use block_n 64 or 128 (got %d)", bn);
  }
  if (bn == 64) return dispatch_epi<K, 64, 1, CG>(e, args, grid, st);
  if (bn == 128) return dispatch_epi<K, 128, 1, CG>(e, args, grid, st);
  if (bn == 256) return dispatch_epi<K, 256, 1, CG>(e, args, grid, st);
  return fail(SVLA_ERR_ARG, "block_n must be 64, 128 or 256 (got %d)", bn);
}

int sm_count() {
  static int counts[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (counts[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    counts[dev] = n;
  }
  return counts[dev];
}

// Tile width.  A k-stage costs about the same time at 64, 128 and 256 columns (measured), so a GEMM takes
// about (rounds of tiles over the SMs) x (k-stages): take the width with the fewest rounds, the wider one on
// a tie (pairs: at most 128 so two accumulator buffers fit TMEM).  When even 64-column tiles leave half of
// the SMs idle, take 64 columns: split-K (which runs on 64-column tiles) then spreads K over the rest.
int choose_block_n(const svla_gemm_desc* d, int sms) {
  const int m_tiles = (d->m + 127) / 128;
  auto tiles = [&](int bn) {
    if (d->pair) return m_tiles * ((d->seg[0].n + bn - 1) / bn);
    int t = 0;
    for (int s = 0; s < d->nseg; ++s) t += (d->seg[s].n + bn - 1) / bn;
    return m_tiles * t;
  };
  if (tiles(64) * 2 <= sms) return 64;
  auto rounds = [&](int bn) { return (tiles(bn) + sms - 1) / sms; };
  int best = 64;
  for (int bn : {128, 256}) {
    if (d->pair && bn > 128) continue;
    if (rounds(bn) <= rounds(best)) best = bn;
  }
  return best;
}

}  // namespace

// the last-error message of the calling thread, for the library's other translation units (engine.cpp)
int32_t set_error(int32_t code, const std::string& msg) {
  t_last_error = msg;
  return code;
}

int32_t run_gemm(const svla_gemm_desc* d, cudaStream_t stream) {
  if (!d) return fail(SVLA_ERR_ARG, "null gemm descriptor");
  if (d->kind < 0 || d->kind > 2) return fail(SVLA_ERR_ARG, "bad operand kind %d", d->kind);
  const Kind kind = static_cast<Kind>(d->kind);
  const Epi epi = static_cast<Epi>(d->epi);
  if (d->m <= 0 || d->k <= 0) return fail(SVLA_ERR_ARG, "bad shape m=%d k=%d", d->m, d->k);
  if (d->nseg < 1 || d->nseg > 3) return fail(SVLA_ERR_ARG, "nseg must be 1..3");
  if (d->pair && d->nseg != 2) return fail(SVLA_ERR_ARG, "a pair needs exactly 2 segments");
  if (epi == Epi::SiluMul && !d->pair) return fail(SVLA_ERR_ARG, "SILU_MUL needs pair = 1");
  if (epi == Epi::I32 && kind != Kind::I8) return fail(SVLA_ERR_ARG, "I32 epilogue needs kind I8");
  if (d->epi < 0 || d->epi > static_cast<int>(Epi::F32)) return fail(SVLA_ERR_ARG, "bad epilogue %d", d->epi);
  {
    // The epilogue moves 16 columns per access (128- or 256-bit vectors): every row it touches must start on a
    // 16-byte boundary, or the launch would fault instead of returning status 1.
    auto al = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; };
    const int out_bytes = (epi == Epi::I32 || epi == Epi::F32) ? 4 : 2;
    int max_n = 0;
    for (int s = 0; s < d->nseg; ++s) {
      const svla_gemm_seg& g = d->seg[s];
      if (g.n > max_n) max_n = g.n;
      if (epi == Epi::Euler) {
        if (g.ldo < g.n) return fail(SVLA_ERR_ARG, "segment %d: EULER row stride %d below n=%d", s, g.ldo, g.n);
        continue;
      }
      if (!g.out) continue;
      if (!al(g.out, 16)) return fail(SVLA_ERR_ARG, "segment %d: output not 16-byte aligned", s);
      if (g.ldo < g.n || (static_cast<long long>(g.ldo) * out_bytes) % 16 != 0)
        return fail(SVLA_ERR_ARG, "segment %d: output row stride %d must be >= n=%d and a multiple of %d", s, g.ldo,
                    g.n, 16 / out_bytes);
    }
    if (epi == Epi::Resid && d->resid &&
        (!al(d->resid, 16) || d->ldr < max_n || d->ldr % 8 != 0))
      return fail(SVLA_ERR_ARG, "RESID: residual must be 16-byte aligned with a row stride >= n and a multiple of 8");
    if (epi == Epi::GeluQuant && d->qout && (!al(d->qout, 16) || d->ldq < max_n || d->ldq % 16 != 0))
      return fail(SVLA_ERR_ARG, "GELU_QUANT: qout must be 16-byte aligned with a row stride >= n and a multiple of 16");
    if (epi == Epi::Euler && d->xt && (!al(d->xt, 4) || !al(d->xt_bf16, 2)))
      return fail(SVLA_ERR_ARG, "EULER: misaligned xt / xt_bf16");
    if (epi == Epi::Rope && d->rope_cs && !al(d->rope_cs, 16))
      return fail(SVLA_ERR_ARG, "ROPE: rope_cs must be 16-byte aligned");
  }
  const int sms = sm_count();
  const int bn = d->block_n ? d->block_n : choose_block_n(d, sms);
  // CTA pairs (256-row tiles over two SMs, half the B rows per SM), on request only: measured on the
  // benchmark's GEMMs they are bit-identical but not faster (SigLIP q/k/v 0.288 -> 0.298 ms, fc1 0.549 ->
  // 0.593 ms, fc2 0.288 -> 0.283 ms, expert down 21.0 -> 22.9 us), so the main loop is not bound by the
  // per-SM operand bytes they save
  if (d->cta_pair < 0 || d->cta_pair > 2) return fail(SVLA_ERR_ARG, "cta_pair must be 0, 1 or 2");
  int cg = 1;
  if (d->cta_pair == 2) {
    if (kind == Kind::W8A16 || bn < 128 || d->split_k > 1 || d->m <= 128 || sms < 2)
      return fail(SVLA_ERR_ARG, "cta_pair 2 needs I8 / BF16 operands, block_n >= 128, no split-K and m > 128");
    cg = 2;
  }
  const int elem_a = (kind == Kind::I8) ? 1 : 2;
  const int elem_b = (kind == Kind::BF16) ? 2 : 1;
  const int bk = (kind == Kind::I8) ? 128 : 64;
  GemmArgs args;
  std::memset(&args, 0, sizeof(args));
  int tiles = 0;
  for (int s = 0; s < d->nseg; ++s) {
    const svla_gemm_seg& g = d->seg[s];
    if (g.n <= 0 || g.n % 16 != 0) return fail(SVLA_ERR_ARG, "segment %d: n=%d must be a positive multiple of 16", s, g.n);
    if (!g.a || !g.b) return fail(SVLA_ERR_ARG, "segment %d: null operand", s);
    if (!g.out && epi != Epi::GeluQuant && epi != Epi::Euler)
      return fail(SVLA_ERR_ARG, "segment %d: null output", s);
    if (g.lda < d->k || g.ldb < d->k) return fail(SVLA_ERR_ARG, "segment %d: lda/ldb smaller than k", s);
    if (epi == Epi::Rope && g.rope && g.n % 64 != 0) return fail(SVLA_ERR_ARG, "RoPE segment n must be a multiple of 64");
    if (kind == Kind::I8 && g.act_scale <= 0.f) return fail(SVLA_ERR_ARG, "segment %d: act_scale must be > 0", s);
    int32_t rc;
    const CUtensorMapDataType dta = (kind == Kind::I8) ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    rc = make_tmap(&args.ta[s], g.a, dta, elem_a, d->k, d->m, g.lda, bk, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc) return rc;
    if (kind == Kind::W8A16) {
      rc = make_tmap(&args.tb[s], g.b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, d->k, g.n, g.ldb, 64, bn,
                     CU_TENSOR_MAP_SWIZZLE_NONE);
    } else {
      const CUtensorMapDataType dtb = (kind == Kind::BF16) ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8;
      rc = make_tmap(&args.tb[s], g.b, dtb, elem_b, d->k, g.n, g.ldb, bk, bn / cg, CU_TENSOR_MAP_SWIZZLE_128B);
    }
    if (rc) return rc;
    GemmSeg& o = args.seg[s];
    o.wscale = g.wscale;
    o.bias = static_cast<const __nv_bfloat16*>(g.bias);
    o.bias_f32 = g.bias_f32;
    o.out = g.out;
    o.ldo = g.ldo;
    o.n = g.n;
    o.tile_begin = d->pair ? 0 : tiles;
    o.act_scale = (kind == Kind::I8) ? g.act_scale : 1.0f;
    o.rope = g.rope;
    if (!d->pair) tiles += (g.n + bn - 1) / bn;
  }
  if (d->pair) {
    if (d->seg[0].n != d->seg[1].n) return fail(SVLA_ERR_ARG, "pair segments must have equal n");
    tiles = (d->seg[0].n + bn - 1) / bn;
  }
  args.nseg = d->nseg;
  args.M = d->m;
  args.K = d->k;
  args.tiles_m = (d->m + 128 * cg - 1) / (128 * cg);
  args.tiles_n = tiles;
  args.rows_per_group = d->rows_per_group;
  args.group_stride = d->group_stride;
  args.row_offset = d->row_offset;
  args.post_scale = d->post_scale;
  args.resid = static_cast<const __nv_bfloat16*>(d->resid);
  args.ldr = d->ldr;
  args.resid_rows = d->resid_rows;
  args.rope_cs = reinterpret_cast<const float2*>(d->rope_cs);
  args.pos = d->pos;
  args.max_pos = d->max_pos;
  args.q_smooth = d->q_smooth;
  args.q_rsmooth = d->q_rsmooth;
  args.q_act = d->q_act;
  args.qout = d->qout;
  args.ldq = d->ldq;
  args.dt = d->dt;
  args.xt = d->xt;
  args.xt_bf16 = static_cast<__nv_bfloat16*>(d->xt_bf16);
  args.err = device_error_ptr();
  args.dbg = reinterpret_cast<unsigned long long*>(d->debug_clock);
  args.weights_resident = d->weights_resident;
  // 256-bit bf16 output stores need every 16-column group of every row 32-byte aligned: base and row stride
  args.out_v8 = 1;
  for (int s = 0; s < d->nseg; ++s)
    if (d->seg[s].out && (reinterpret_cast<uintptr_t>(d->seg[s].out) % 32 != 0 || d->seg[s].ldo % 16 != 0)) args.out_v8 = 0;
  args.resid_v8 = (d->resid && reinterpret_cast<uintptr_t>(d->resid) % 32 == 0 && d->ldr % 16 == 0) ? 1 : 0;
  // a pair over one A operand (the expert's gate / up on the same normalised rows): one MMA of N = 2 * BN
  // per k-step instead of two of N = BN -- the tensor core takes about as long to issue either
  args.shared_a = (d->pair && cg == 1 && kind != Kind::W8A16 && 2 * bn <= 256 && d->seg[0].a == d->seg[1].a &&
                   d->seg[0].lda == d->seg[1].lda) ? 1 : 0;
  if (epi == Epi::Resid && !d->resid) return fail(SVLA_ERR_ARG, "RESID needs a residual");
  if (epi == Epi::Rope && (!d->rope_cs || !d->pos || d->max_pos <= 0)) return fail(SVLA_ERR_ARG, "ROPE needs rope_cs/pos");
  if (epi == Epi::GeluQuant && d->qout && (!d->q_smooth || d->q_act <= 0.f))
    return fail(SVLA_ERR_ARG, "GELU_QUANT with qout needs q_smooth and q_act > 0");
  if (epi == Epi::GeluQuant && !d->qout && !d->seg[0].out) return fail(SVLA_ERR_ARG, "GELU_QUANT needs qout or out");
  if (epi == Epi::Euler && (!d->xt || !d->xt_bf16)) return fail(SVLA_ERR_ARG, "EULER needs xt/xt_bf16");
  // split-K (see svla_gemm_desc): only with a workspace, 64-column tiles and few output tiles
  const long long out_tiles = static_cast<long long>(args.tiles_m) * args.tiles_n;
  const int kstage = kind == Kind::I8 ? 128 : 64;  // K elements per pipeline stage
  const int k_tiles = (d->k + kstage - 1) / kstage;
  args.splits = 1;
  args.kt_per_split = k_tiles;
  if (d->split_k < 0) return fail(SVLA_ERR_ARG, "split_k must be >= 0");
  if (d->split_k > 1 && !d->workspace) return fail(SVLA_ERR_ARG, "split_k needs a workspace");
  if (d->split_k > 1 && bn != 64) return fail(SVLA_ERR_ARG, "split_k needs block_n 64 (got %d)", bn);
  if (d->workspace && d->split_k != 1 && bn == 64) {
    if (reinterpret_cast<uintptr_t>(d->workspace) % 256 != 0) return fail(SVLA_ERR_ARG, "workspace not 256-byte aligned");
    // automatic: up to 4 splits (the last split reads every split's partial: more splits cost more than
    // the shorter K loop saves), at least 4 k-tiles each, within the SMs the output tiles leave free
    long long want = 1;
    if (d->split_k > 1) {
      want = d->split_k;
    } else if (out_tiles * 2 <= sms) {
      want = k_tiles / 4;
      if (want > 4) want = 4;
      if (want > sms / out_tiles) want = sms / out_tiles;
      if (want < 1) want = 1;
    }
    if (want > k_tiles) want = k_tiles;
    if (want > 32) want = 32;
    const long long per_split = static_cast<long long>(d->pair ? 2 : 1) * 128 * bn * 4;
    const long long room = static_cast<long long>(d->workspace_bytes) - SVLA_SPLITK_COUNTER_BYTES;
    if (want > 1 && (out_tiles > SVLA_SPLITK_COUNTER_BYTES / 4 || room < out_tiles * per_split * want)) {
      if (d->split_k > 1)
        return fail(SVLA_ERR_ARG, "split_k=%d does not fit the workspace (%zu bytes)", d->split_k, d->workspace_bytes);
      want = (out_tiles <= SVLA_SPLITK_COUNTER_BYTES / 4 && room > 0) ? room / (out_tiles * per_split) : 1;
      if (want < 1) want = 1;
    }
    if (want > 1) {
      const int kps = static_cast<int>((k_tiles + want - 1) / want);
      args.splits = (k_tiles + kps - 1) / kps;  // every split has at least one k-tile
      args.kt_per_split = kps;
      args.counters = static_cast<int*>(d->workspace);
      args.partial = reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(d->workspace) + SVLA_SPLITK_COUNTER_BYTES);
    }
  }
  const long long total_tiles = out_tiles * args.splits;
  const long long units = sms / cg;  // CTAs (pairs) resident at once, one per SM (pair of SMs)
  dim3 grid(static_cast<unsigned>(cg * (total_tiles < units ? total_tiles : units)));
  if (cg == 2) {
    if (args.splits > 1) return fail(SVLA_ERR_ARG, "CTA pairs do not split K");
    switch (kind) {
      case Kind::I8: return dispatch_bn<Kind::I8, 2>(bn, d->pair, epi, args, grid, stream);
      case Kind::BF16: return dispatch_bn<Kind::BF16, 2>(bn, d->pair, epi, args, grid, stream);
      default: return fail(SVLA_ERR_ARG, "CTA pairs take I8 / BF16 operands");
    }
  }
  switch (kind) {
    case Kind::I8: return dispatch_bn<Kind::I8, 1>(bn, d->pair, epi, args, grid, stream);
    case Kind::BF16: return dispatch_bn<Kind::BF16, 1>(bn, d->pair, epi, args, grid, stream);
    case Kind::W8A16: return dispatch_bn<Kind::W8A16, 1>(bn, d->pair, epi, args, grid, stream);
  }
  return fail(SVLA_ERR_ARG, "unreachable");
}

}  // namespace svla

using namespace svla;

static inline cudaStream_t cs(svla_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

extern "C" {

const char* svla_last_error(void) { return t_last_error.c_str(); }

const char* svla_version(void) {
  return "svla 0.2 sm_100a (tcgen05 kind::i8 / kind::f16 GEMMs with split-K, tcgen05 + mma.sync attention, TMA)";
}

int32_t svla_device_error(int32_t* code, int32_t reset) {
  int* p = device_error_ptr();
  if (!p) return fail(SVLA_ERR_CUDA, "device error word unavailable");
  int v = 0;
  if (cudaMemcpy(&v, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
    return fail(SVLA_ERR_CUDA, "reading the device error word failed");
  if (code) *code = v;
  if (reset) {
    int z = 0;
    if (cudaMemcpy(p, &z, sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess)
      return fail(SVLA_ERR_CUDA, "clearing the device error word failed");
  }
  return SVLA_OK;
}

int32_t svla_pack_weight_i8(const void* weight, const float* smooth, int32_t n, int32_t k, int8_t* qweight,
                            float* wscale, svla_stream_t stream) {
  if (!weight || !qweight || !wscale || n <= 0 || k <= 0) return fail(SVLA_ERR_ARG, "svla_pack_weight_i8: bad args");
  return launch(pack_weight_kernel, dim3(n), dim3(256), 0, cs(stream), "pack_weight_kernel", static_cast<const __nv_bfloat16*>(weight), k, smooth, qweight, wscale);
}

int32_t svla_dequant_weight_bf16(const int8_t* qweight, const float* wscale, int32_t n, int32_t k, void* out,
                                 svla_stream_t stream) {
  if (!qweight || !wscale || !out || n <= 0 || k <= 0 || k % 8)
    return fail(SVLA_ERR_ARG, "svla_dequant_weight_bf16: bad args (k must be a multiple of 8)");
  const long long groups = static_cast<long long>(n) * k / 8;
  return launch(dequant_weight_kernel, dim3(static_cast<unsigned>((groups + 255) / 256)), dim3(256), 0, cs(stream),
                "dequant_weight_kernel", qweight, wscale, n, k, static_cast<__nv_bfloat16*>(out));
}

int32_t svla_quantize_smooth(const void* x, int32_t ldx, const float* smooth, float act_scale, int8_t* q, int32_t ldq,
                             int32_t m, int32_t k, svla_stream_t stream) {
  if (!x || !q || m <= 0 || k <= 0 || k % 8 || ldx % 8 || ldq % 8 || ldx < k || ldq < k || !(act_scale > 0.f))
    return fail(SVLA_ERR_ARG, "svla_quantize_smooth: bad args (k, ldx >= k, ldq >= k must be multiples of 8)");
  // each thread loads 8 bf16 values (16 bytes) and stores 8 int8 values (8 bytes)
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 || reinterpret_cast<uintptr_t>(q) % 8 != 0)
    return fail(SVLA_ERR_ARG, "svla_quantize_smooth: x must be 16-byte and q 8-byte aligned");
  const long long total = static_cast<long long>(m) * (k / 8);
  return launch(smooth_quant_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, cs(stream), "smooth_quant_kernel",
                static_cast<const __nv_bfloat16*>(x), ldx, smooth, act_scale, q, ldq, m, k);
}

int32_t svla_channel_percentile(const void* x, int64_t ldx, int32_t calls, int32_t rows, int32_t k, float q,
                                float* amax, float* pamax, svla_stream_t stream) {
  if (!x || !amax || !pamax || k <= 0 || ldx < k || rows < 1 || rows > kPctMaxRows || calls < 1 || calls > 65535 ||
      !(q >= 0.f && q <= 1.f))
    return fail(SVLA_ERR_ARG, "svla_channel_percentile: bad args (1 <= rows <= %d, 1 <= calls <= 65535, ldx >= k, "
                "0 <= q <= 1)", kPctMaxRows);
  if (reinterpret_cast<uintptr_t>(x) % 2 || reinterpret_cast<uintptr_t>(amax) % 4 ||
      reinterpret_cast<uintptr_t>(pamax) % 4)
    return fail(SVLA_ERR_ARG, "svla_channel_percentile: misaligned x / amax / pamax");
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(SVLA_ERR_ARG, "device index %d out of range", dev);
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(channel_percentile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(percentile_smem(kPctMaxRows)));
    if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  // torch.quantile's interpolation point, in fp32 as torch computes it for an fp32 input
  const float rank = q * static_cast<float>(rows - 1);
  PercentileArgs a;
  a.x = static_cast<const __nv_bfloat16*>(x);
  a.ldx = ldx;
  a.calls = calls;
  a.rows = rows;
  a.K = k;
  a.lo = static_cast<int>(std::floor(rank));
  a.hi = static_cast<int>(std::ceil(rank));
  a.w = rank - static_cast<float>(a.lo);
  a.amax = amax;
  a.pamax = pamax;
  return launch(channel_percentile_kernel, dim3(static_cast<unsigned>((k + kPctCols - 1) / kPctCols), calls),
                dim3(kPctCols * 32), percentile_smem(rows), cs(stream), "channel_percentile_kernel", a);
}

int32_t svla_gemm(const svla_gemm_desc* desc, svla_stream_t stream) { return run_gemm(desc, cs(stream)); }

int32_t svla_gemm_i8_i32(const int8_t* qx, const int8_t* qw, int32_t m, int32_t n, int32_t k, int32_t* acc,
                         svla_stream_t stream) {
  svla_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.kind = SVLA_KIND_I8;
  d.epi = SVLA_EPI_I32;
  d.m = m;
  d.k = k;
  d.nseg = 1;
  d.seg[0].a = qx;
  d.seg[0].lda = k;
  d.seg[0].b = qw;
  d.seg[0].ldb = k;
  d.seg[0].out = acc;
  d.seg[0].ldo = n;
  d.seg[0].n = n;
  d.seg[0].act_scale = 1.0f;
  return run_gemm(&d, cs(stream));
}

size_t svla_sq_linear_w8a8_workspace_size(int32_t m, int32_t k) {
  return (static_cast<size_t>(m) * k + 255) / 256 * 256;
}

int32_t svla_sq_linear_w8a8(const void* x, const float* smooth, float act_scale, const int8_t* qweight,
                            const float* wscale, const void* bias, int32_t m, int32_t n, int32_t k, void* y,
                            void* workspace, size_t workspace_bytes, svla_stream_t stream) {
  if (!workspace || workspace_bytes < svla_sq_linear_w8a8_workspace_size(m, k))
    return fail(SVLA_ERR_ARG, "svla_sq_linear_w8a8: workspace too small (%zu < %zu)", workspace_bytes,
                svla_sq_linear_w8a8_workspace_size(m, k));
  int8_t* qx = static_cast<int8_t*>(workspace);
  int32_t rc = svla_quantize_smooth(x, k, smooth, act_scale, qx, k, m, k, stream);
  if (rc) return rc;
  svla_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.kind = SVLA_KIND_I8;
  d.epi = SVLA_EPI_BF16;
  d.m = m;
  d.k = k;
  d.nseg = 1;
  d.seg[0] = svla_gemm_seg{qx, k, qweight, k, wscale, bias, nullptr, y, n, n, act_scale, 0};
  return run_gemm(&d, cs(stream));
}

int32_t svla_w8a16_linear(const void* x, const int8_t* qweight, const float* wscale, const void* bias, int32_t m,
                          int32_t n, int32_t k, void* y, svla_stream_t stream) {
  svla_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.kind = SVLA_KIND_W8A16;
  d.epi = SVLA_EPI_BF16;
  d.m = m;
  d.k = k;
  d.nseg = 1;
  d.seg[0] = svla_gemm_seg{x, k, qweight, k, wscale, bias, nullptr, y, n, n, 1.0f, 0};
  return run_gemm(&d, cs(stream));
}

int32_t svla_norm_quant(const svla_norm_desc* d, svla_stream_t stream) {
  if (!d || !d->x || !d->weight || d->m <= 0 || d->k <= 0) return fail(SVLA_ERR_ARG, "svla_norm_quant: bad args");
  if (d->k % 8 || d->ldx % 8 || (d->y && d->ldy % 8) || (d->nq && d->ldq % 8))
    return fail(SVLA_ERR_ARG, "svla_norm_quant: k and row strides must be multiples of 8");
  if (d->nq < 0 || d->nq > 3) return fail(SVLA_ERR_ARG, "svla_norm_quant: nq must be 0..3");
  if (d->layernorm && !d->bias) return fail(SVLA_ERR_ARG, "svla_norm_quant: LayerNorm needs a bias");
  if (d->pixel_shuffle && (d->ps_grid % d->pixel_shuffle || d->m % (d->ps_grid * d->ps_grid)))
    return fail(SVLA_ERR_ARG, "svla_norm_quant: pixel shuffle grid mismatch");
  NormQuantArgs a;
  std::memset(&a, 0, sizeof(a));
  a.x = static_cast<const __nv_bfloat16*>(d->x);
  a.ldx = d->ldx;
  a.w = static_cast<const __nv_bfloat16*>(d->weight);
  a.b = static_cast<const __nv_bfloat16*>(d->bias);
  a.eps = d->eps;
  a.M = d->m;
  a.K = d->k;
  a.y = static_cast<__nv_bfloat16*>(d->y);
  a.ldy = d->ldy;
  a.nq = d->nq;
  for (int i = 0; i < 3; ++i) {
    a.q[i] = d->q[i];
    a.smooth[i] = d->smooth[i];
    a.rsmooth[i] = d->rsmooth[i];
    a.act[i] = d->act[i];
    if (i < d->nq && (!d->q[i] || !d->smooth[i] || d->act[i] <= 0.f))
      return fail(SVLA_ERR_ARG, "svla_norm_quant: quant output %d incomplete", i);
  }
  a.ldq = d->ldq;
  a.pixel_shuffle = d->pixel_shuffle;
  a.ps_grid = d->ps_grid;
  const int nv = (d->k + 255) / 256;
  // 8 rows per 256-thread block at most; at most 8 blocks per SM resident at once, each warp then
  // streams several rows
  const long long max_blocks = static_cast<long long>(sm_count()) * 8;
  const unsigned blocks = static_cast<unsigned>(((d->m + 7) / 8) < max_blocks ? (d->m + 7) / 8 : max_blocks);
  cudaStream_t st = cs(stream);
#define SVLA_NORM(NV)                                                                                     \
  if (nv <= NV) {                                                                                         \
    if (d->layernorm) return launch(norm_quant_kernel<NV, true>, dim3(blocks), dim3(256), 0, st, "norm_quant_kernel", a); \
    return launch(norm_quant_kernel<NV, false>, dim3(blocks), dim3(256), 0, st, "norm_quant_kernel", a);  \
  }
  SVLA_NORM(3)
  SVLA_NORM(4)
  SVLA_NORM(12)
#undef SVLA_NORM
  return fail(SVLA_ERR_ARG, "svla_norm_quant: k=%d too large (max 3072)", d->k);
}

// 3-D bf16 tensor map (column, row, batch) with a 64 x box_rows x 1 box and the 128-byte swizzle; rows past
// `rows` (of each batch) read as zeros
static int32_t make_tmap_bhd(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows, uint64_t batch,
                             uint64_t rs, uint64_t bs, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SVLA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {cols, rows, batch};
  cuuint64_t strides[2] = {rs * 2, bs * 2};
  cuuint32_t box[3] = {64, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVLA_ERR_ARG, "cuTensorMapEncodeTiled (3-D) failed (%d)", static_cast<int>(r));
  return SVLA_OK;
}

// 4-D bf16 tensor map of Q [batch][query][head][64] (dim, head, query, batch) with a 64 x G x QT x 1 box and the
// 128-byte swizzle: one box is the packed rows (query-major, then head) of a kv head's G query heads
static int32_t make_tmap_q4(CUtensorMap* map, const void* base, uint64_t heads, uint64_t lq, uint64_t batch,
                            uint64_t rs, uint64_t bs, uint32_t g, uint32_t qt) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(SVLA_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[4] = {64, heads, lq, batch};
  cuuint64_t strides[3] = {128, rs * 2, bs * 2};
  cuuint32_t box[4] = {64, g, qt, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(SVLA_ERR_ARG, "cuTensorMapEncodeTiled (4-D) failed (%d)", static_cast<int>(r));
  return SVLA_OK;
}

}  // extern "C"

template <int MASK>
static int32_t launch_attention_tc(const AttnTcArgs& a, dim3 grid, cudaStream_t stream) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(SVLA_ERR_ARG, "device index %d out of range", dev);
  auto kern = attention_tc_kernel<MASK>;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, atc::kSmemBytes);
    if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  return launch(kern, grid, dim3(atc::kThreads), atc::kSmemBytes, stream, "attention_tc_kernel", a);
}

extern "C" {

static int32_t run_attention_tc(const svla_attn_desc* d, float scale, cudaStream_t stream) {
  AttnTcArgs a;
  std::memset(&a, 0, sizeof(a));
  const int g = d->hq / d->hkv, qt = 128 / g;
  int32_t rc = make_tmap_q4(&a.tq, d->q, d->hq, d->lq, d->batch, d->q_rs, d->q_bs, g, qt);
  if (rc) return rc;
  rc = make_tmap_bhd(&a.tk, d->k1, static_cast<uint64_t>(d->hkv) * 64, d->l1, d->batch, d->kv1_rs, d->kv1_bs,
                     atc::kKeys);
  if (rc) return rc;
  rc = make_tmap_bhd(&a.tv, d->v1, static_cast<uint64_t>(d->hkv) * 64, d->l1, d->batch, d->kv1_rs, d->kv1_bs,
                     atc::kKeys);
  if (rc) return rc;
  if (d->l2 > 0) {
    rc = make_tmap_bhd(&a.tk2, d->k2, static_cast<uint64_t>(d->hkv) * 64, d->l2, d->batch, d->kv2_rs, d->kv2_bs,
                       atc::kKeys);
    if (rc) return rc;
    rc = make_tmap_bhd(&a.tv2, d->v2, static_cast<uint64_t>(d->hkv) * 64, d->l2, d->batch, d->kv2_rs, d->kv2_bs,
                       atc::kKeys);
    if (rc) return rc;
  }
  a.mask = d->mask;
  a.mask_bs = d->mask_bs;
  a.mask_rs = d->mask_rs;
  a.key_mask = d->key_mask;
  a.key_mask_bs = d->key_mask_bs;
  a.mask_keys = d->mask_keys;
  a.o = static_cast<__nv_bfloat16*>(d->o);
  a.o_bs = d->o_bs;
  a.o_rs = d->o_rs;
  a.qo = d->qo;
  a.qo_bs = d->qo_bs;
  a.qo_rs = d->qo_rs;
  a.qo_smooth = d->qo_smooth;
  a.qo_rsmooth = d->qo_rsmooth;
  a.qo_act = d->qo_act;
  a.Lq = d->lq;
  a.L1 = d->l1;
  a.L2 = d->l2 > 0 ? d->l2 : 0;
  a.Hq = d->hq;
  a.Hkv = d->hkv;
  a.G = g;
  a.QT = qt;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.dbg = static_cast<unsigned long long*>(d->debug_clock);
  a.err = device_error_ptr();
  // one 128-row tile per CTA, two CTAs per SM: one CTA's exponentials fill the other's gaps, and one CTA's
  // set-up and epilogue overlap the other's key loop
  dim3 grid(static_cast<unsigned>((d->lq + qt - 1) / qt), d->hkv, d->batch);
  if (d->key_mask) return launch_attention_tc<kTcMaskStructured>(a, grid, stream);
  if (d->mask) return launch_attention_tc<kTcMaskBytes>(a, grid, stream);
  return launch_attention_tc<kTcMaskNone>(a, grid, stream);
}

int32_t svla_attention(const svla_attn_desc* d, svla_stream_t stream) {
  if (!d || !d->q || !d->k1 || !d->v1 || d->batch <= 0 || d->lq <= 0 || d->l1 <= 0 || d->hq <= 0 || d->hkv <= 0)
    return fail(SVLA_ERR_ARG, "svla_attention: bad args");
  if (d->hq % d->hkv) return fail(SVLA_ERR_ARG, "svla_attention: hq must be a multiple of hkv");
  if (d->l2 > 0 && (!d->k2 || !d->v2)) return fail(SVLA_ERR_ARG, "svla_attention: second key source missing");
  if (!d->o && !d->qo) return fail(SVLA_ERR_ARG, "svla_attention: no output");
  if (d->qo && (!d->qo_smooth || d->qo_act <= 0.f)) return fail(SVLA_ERR_ARG, "svla_attention: qo needs smooth/act");
  if ((d->q_rs % 8) || (d->kv1_rs % 8) || (d->l2 > 0 && d->kv2_rs % 8))
    return fail(SVLA_ERR_ARG, "svla_attention: row strides must be multiples of 8");
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.q = static_cast<const __nv_bfloat16*>(d->q);
  a.q_bs = d->q_bs;
  a.q_rs = d->q_rs;
  a.k1 = static_cast<const __nv_bfloat16*>(d->k1);
  a.v1 = static_cast<const __nv_bfloat16*>(d->v1);
  a.kv1_bs = d->kv1_bs;
  a.kv1_rs = d->kv1_rs;
  a.L1 = d->l1;
  a.k2 = static_cast<const __nv_bfloat16*>(d->k2);
  a.v2 = static_cast<const __nv_bfloat16*>(d->v2);
  a.kv2_bs = d->kv2_bs;
  a.kv2_rs = d->kv2_rs;
  a.L2 = d->l2 > 0 ? d->l2 : 0;
  a.mask = d->mask;
  a.mask_bs = d->mask_bs;
  a.mask_rs = d->mask_rs;
  if (d->key_mask && d->mask) return fail(SVLA_ERR_ARG, "svla_attention: give mask or key_mask, not both");
  if (d->key_mask && (d->mask_keys <= 0 || d->mask_keys > d->l1 + (d->l2 > 0 ? d->l2 : 0)))
    return fail(SVLA_ERR_ARG, "svla_attention: mask_keys must be in 1..l1+l2");
  a.key_mask = d->key_mask;
  a.key_mask_bs = d->key_mask_bs;
  a.mask_keys = d->mask_keys;
  a.o = static_cast<__nv_bfloat16*>(d->o);
  a.o_bs = d->o_bs;
  a.o_rs = d->o_rs;
  a.qo = d->qo;
  a.qo_bs = d->qo_bs;
  a.qo_rs = d->qo_rs;
  a.qo_smooth = d->qo_smooth;
  a.qo_rsmooth = d->qo_rsmooth;
  a.qo_act = d->qo_act;
  a.Lq = d->lq;
  a.Hq = d->hq;
  a.Hkv = d->hkv;
  a.scale = d->scale > 0.f ? d->scale : 0.125f;
  const bool a16 = [&] {
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    return al(d->q) && al(d->k1) && al(d->v1) && (!d->o || (al(d->o) && d->o_rs % 8 == 0 && d->o_bs % 8 == 0)) &&
           (!d->qo || (al(d->qo) && d->qo_rs % 16 == 0 && d->qo_bs % 16 == 0)) && d->q_bs % 8 == 0 &&
           d->kv1_bs % 8 == 0 && (!d->qo_rsmooth || al(d->qo_rsmooth));
  }();
  // the tcgen05 kernel reads Q / K / V through tensor maps (16-byte aligned bases and strides), a byte mask as
  // aligned 16-key runs of rows padded to a multiple of 16 keys (single key source), key flags as aligned runs
  const bool tc_ok = [&] {
    auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!a16 || d->hq / d->hkv > 128) return false;
    if (d->l2 > 0 && (!al(d->k2) || !al(d->v2) || d->kv2_rs % 8 || d->kv2_bs % 8)) return false;
    if (d->mask && (d->l2 > 0 || !al(d->mask) || d->mask_rs % 16 || d->mask_bs % 16 ||
                    d->mask_rs < ((d->l1 + 15) & ~15)))
      return false;
    if (d->key_mask && (!al(d->key_mask) || d->key_mask_bs % 16)) return false;
    return true;
  }();
  if (d->impl == SVLA_ATTN_TCGEN05 && !tc_ok)
    return fail(SVLA_ERR_ARG, "svla_attention: the tcgen05 kernel needs 16-byte aligned operands and strides, "
                              "byte masks on a single key source with rows padded to 16 keys");
  // automatic choice: the tcgen05 kernel for unmasked calls (the SigLIP encoder: 809 vs 1668 us at 128 images);
  // masked calls stay on the mma.sync kernel, which measured as fast or faster at the path's masked shapes
  // (expert self 35.3 vs 33.8 us, cross 28.8 vs 29.5 us, text prefix 76.4 vs 92.5 us at batch 64): a CTA there
  // holds 3-4 key tiles, too few to amortise the tensor-memory setup, and GQA rows fill 128-row tiles unevenly
  const bool masked = d->mask || d->key_mask;
  if (tc_ok && (d->impl == SVLA_ATTN_TCGEN05 || (d->impl == SVLA_ATTN_AUTO && !masked)))
    return run_attention_tc(d, a.scale, cs(stream));
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(SVLA_ERR_ARG, "device index %d out of range", dev);
  const int smem = static_cast<int>(sizeof(attn_detail::Smem));
  if (!configured[dev]) {
    for (auto kern : {attention_kernel<attn_detail::kMaskNone>, attention_kernel<attn_detail::kMaskBytes>,
                      attention_kernel<attn_detail::kMaskStructured>}) {
      cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    configured[dev] = true;
  }
  // packed rows of one kv head (its query heads' queries) split into equal tiles of 16 x warps rows
  const long long rows = static_cast<long long>(d->hq / d->hkv) * d->lq;
  const long long tiles = (rows + attn_detail::kRows - 1) / attn_detail::kRows;
  if (tiles > 65535) return fail(SVLA_ERR_ARG, "svla_attention: too many query rows");
  a.rows = static_cast<int>(((rows + tiles - 1) / tiles + 15) / 16 * 16);
  dim3 grid(static_cast<unsigned>(tiles), d->hkv, d->batch);
  if (a.key_mask)
    return launch(attention_kernel<attn_detail::kMaskStructured>, dim3(grid), dim3(a.rows * 2), smem, cs(stream),
                  "attention_kernel", a);
  if (a.mask)
    return launch(attention_kernel<attn_detail::kMaskBytes>, dim3(grid), dim3(a.rows * 2), smem, cs(stream),
                  "attention_kernel", a);
  return launch(attention_kernel<attn_detail::kMaskNone>, dim3(grid), dim3(a.rows * 2), smem, cs(stream),
                "attention_kernel", a);
}

int32_t svla_rope_layout(const void* q_raw, const void* k_raw, const int32_t* pos, void* q_out, void* k_out,
                         int32_t batch, int32_t seq_len, int32_t q_heads, int32_t kv_heads, float max_wavelength,
                         svla_stream_t stream) {
  const svla_rope_params p{q_heads, kv_heads, 64, max_wavelength};
  return svla_fused_rope_layout(q_raw, k_raw, pos, q_out, k_out, batch, seq_len, &p, SVLA_DT_BF16, SVLA_DT_INT32,
                                stream);
}

}  // extern "C"

namespace {

int32_t check_rope_params(const svla_rope_params* p, int32_t batch, int32_t seq_len, const char* who) {
  if (!p) return fail(SVLA_ERR_ARG, "%s: null params", who);
  if (batch <= 0 || seq_len <= 0 || p->q_heads <= 0 || p->kv_heads <= 0 || p->q_heads % p->kv_heads != 0 ||
      p->head_dim <= 0 || p->head_dim % 2 != 0 || !(p->max_wavelength > 0.f))
    return fail(SVLA_ERR_ARG, "%s: bad shape or params (batch %d, seq_len %d, heads %d/%d, head_dim %d)", who, batch,
                seq_len, p->q_heads, p->kv_heads, p->head_dim);
  return SVLA_OK;
}

template <typename T, typename PosT>
int32_t launch_rope_layout_t(const void* q, const void* k, const void* pos, void* qo, void* ko, int32_t B, int32_t L,
                             const svla_rope_params& p, cudaStream_t st) {
  const long long total = static_cast<long long>(B) * L * (p.q_heads + p.kv_heads) * (p.head_dim / 2);
  return launch(rope_layout_kernel<T, PosT>, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, st,
                "rope_layout_kernel", static_cast<const T*>(q), static_cast<const T*>(k),
                static_cast<const PosT*>(pos), static_cast<T*>(qo), static_cast<T*>(ko), static_cast<int>(B),
                static_cast<int>(L), p.q_heads, p.kv_heads, p.head_dim, p.max_wavelength);
}

template <typename T>
int32_t launch_rope_layout_pos(int32_t pos_type, const void* q, const void* k, const void* pos, void* qo, void* ko,
                               int32_t B, int32_t L, const svla_rope_params& p, cudaStream_t st) {
  if (pos_type == SVLA_DT_INT32) return launch_rope_layout_t<T, int32_t>(q, k, pos, qo, ko, B, L, p, st);
  if (pos_type == SVLA_DT_INT64) return launch_rope_layout_t<T, long long>(q, k, pos, qo, ko, B, L, p, st);
  return fail(SVLA_ERR_ARG, "svla_fused_rope_layout: position type %d (int32 %d or int64 %d)", pos_type,
              SVLA_DT_INT32, SVLA_DT_INT64);
}

template <typename T, typename PosT>
int32_t launch_rope_attention_t(const RopeAttnArgs& a, cudaStream_t st) {
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(SVLA_ERR_ARG, "device index %d out of range", dev);
  auto kern = rope_attention_kernel<T, PosT>;
  const size_t smem = rope_attention_smem();
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>((a.L + a.qpc - 1) / a.qpc), a.Hkv, a.B);
  return launch(kern, grid, dim3(kRopeAttnWarps * 32), smem, st, "rope_attention_kernel", a);
}

template <typename T>
int32_t launch_rope_attention_pos(int32_t pos_type, const RopeAttnArgs& a, cudaStream_t st) {
  if (a.pos == nullptr || pos_type == SVLA_DT_INT32) return launch_rope_attention_t<T, int32_t>(a, st);
  if (pos_type == SVLA_DT_INT64) return launch_rope_attention_t<T, long long>(a, st);
  return fail(SVLA_ERR_ARG, "svla_fused_rope_attention: position type %d (int32 %d or int64 %d)", pos_type,
              SVLA_DT_INT32, SVLA_DT_INT64);
}

int32_t run_rope_attention(const void* q, const void* k, const void* v, const void* pos, const void* mask,
                           int mask_f32, float* ctx, int32_t B, int32_t L, const svla_rope_params* p, int32_t data_type,
                           int32_t pos_type, cudaStream_t st, const char* who) {
  int32_t rc = check_rope_params(p, B, L, who);
  if (rc) return rc;
  if (!q || !k || !v || !ctx) return fail(SVLA_ERR_ARG, "%s: null q, k, v or context", who);
  if (p->head_dim % 32 != 0 || p->head_dim > kRopeAttnMaxD)
    return fail(SVLA_ERR_ARG, "%s: head_dim %d must be a multiple of 32 up to %d", who, p->head_dim, kRopeAttnMaxD);
  const int g = p->q_heads / p->kv_heads;
  if (g > kRopeAttnRows) return fail(SVLA_ERR_ARG, "%s: more than %d query heads per kv head", who, kRopeAttnRows);
  RopeAttnArgs a{};
  a.q = q;
  a.k = k;
  a.v = v;
  a.pos = pos;
  a.mask = mask;
  a.mask_f32 = mask_f32;
  a.ctx = ctx;
  a.B = B;
  a.L = L;
  a.Hq = p->q_heads;
  a.Hkv = p->kv_heads;
  a.D = p->head_dim;
  a.qpc = kRopeAttnRows / g;
  a.max_wavelength = p->max_wavelength;
  a.scale = 1.0f / std::sqrt(static_cast<float>(p->head_dim));
  switch (data_type) {
    case SVLA_DT_FLOAT: return launch_rope_attention_pos<float>(pos_type, a, st);
    case SVLA_DT_HALF: return launch_rope_attention_pos<__half>(pos_type, a, st);
    case SVLA_DT_BF16: return launch_rope_attention_pos<__nv_bfloat16>(pos_type, a, st);
    default: return fail(SVLA_ERR_ARG, "%s: data type %d (float %d, half %d or bf16 %d)", who, data_type,
                         SVLA_DT_FLOAT, SVLA_DT_HALF, SVLA_DT_BF16);
  }
}

}  // namespace

extern "C" {

int32_t svla_fused_rope_layout(const void* q_raw, const void* k_raw, const void* position_ids, void* q_out,
                               void* k_out, int32_t batch, int32_t seq_len, const svla_rope_params* params,
                               int32_t data_type, int32_t position_type, svla_stream_t stream) {
  int32_t rc = check_rope_params(params, batch, seq_len, "svla_fused_rope_layout");
  if (rc) return rc;
  if (!q_raw || !k_raw || !position_ids || !q_out || !k_out)
    return fail(SVLA_ERR_ARG, "svla_fused_rope_layout: null pointer argument");
  const svla_rope_params& p = *params;
  switch (data_type) {
    case SVLA_DT_FLOAT:
      return launch_rope_layout_pos<float>(position_type, q_raw, k_raw, position_ids, q_out, k_out, batch, seq_len, p,
                                           cs(stream));
    case SVLA_DT_HALF:
      return launch_rope_layout_pos<__half>(position_type, q_raw, k_raw, position_ids, q_out, k_out, batch, seq_len,
                                            p, cs(stream));
    case SVLA_DT_BF16:
      return launch_rope_layout_pos<__nv_bfloat16>(position_type, q_raw, k_raw, position_ids, q_out, k_out, batch,
                                                   seq_len, p, cs(stream));
    default:
      return fail(SVLA_ERR_ARG, "svla_fused_rope_layout: data type %d (float %d, half %d or bf16 %d)", data_type,
                  SVLA_DT_FLOAT, SVLA_DT_HALF, SVLA_DT_BF16);
  }
}

int32_t svla_fused_rope_attention(const void* q_raw, const void* k_raw, const void* v_raw, const void* position_ids,
                                  const void* mask, float* context, int32_t batch, int32_t seq_len,
                                  const svla_rope_params* params, int32_t data_type, int32_t position_type,
                                  svla_stream_t stream) {
  if (!position_ids || !mask) return fail(SVLA_ERR_ARG, "svla_fused_rope_attention: null positions or mask");
  return run_rope_attention(q_raw, k_raw, v_raw, position_ids, mask, 0, context, batch, seq_len, params, data_type,
                            position_type, cs(stream), "svla_fused_rope_attention");
}

int32_t svla_fused_rope_attention_f32_mask_implicit_pos(const float* q_raw, const float* k_raw, const float* v_raw,
                                                        const float* mask, float* context, int32_t batch,
                                                        int32_t seq_len, const svla_rope_params* params,
                                                        svla_stream_t stream) {
  if (!mask) return fail(SVLA_ERR_ARG, "svla_fused_rope_attention_f32_mask_implicit_pos: null mask");
  return run_rope_attention(q_raw, k_raw, v_raw, nullptr, mask, 1, context, batch, seq_len, params, SVLA_DT_FLOAT,
                            SVLA_DT_INT32, cs(stream), "svla_fused_rope_attention_f32_mask_implicit_pos");
}

int32_t svla_resize_pad_images(const void* src, int32_t src_u8_hwc, int32_t n, int32_t c, int32_t h, int32_t w,
                               float* out, int64_t out_image_stride, int32_t out_h, int32_t out_w, float pad_value,
                               svla_stream_t stream) {
  if (!src || !out || n <= 0 || c <= 0 || h <= 0 || w <= 0 || out_h <= 0 || out_w <= 0 ||
      out_image_stride < static_cast<int64_t>(c) * out_h * out_w)
    return fail(SVLA_ERR_ARG, "svla_resize_pad_images: bad args");
  ResizeArgs a;
  a.src = src;
  a.u8_hwc = src_u8_hwc ? 1 : 0;
  a.N = n;
  a.C = c;
  a.H = h;
  a.W = w;
  // the aspect-preserving size, in double precision like the Python reference (int() truncation)
  const double ratio = std::max(static_cast<double>(w) / out_w, static_cast<double>(h) / out_h);
  a.rh = static_cast<int>(h / ratio);
  a.rw = static_cast<int>(w / ratio);
  if (a.rh <= 0 || a.rw <= 0 || a.rh > out_h || a.rw > out_w) return fail(SVLA_ERR_ARG, "svla_resize_pad_images: degenerate size");
  a.OH = out_h;
  a.OW = out_w;
  a.pad_value = pad_value;
  a.out = out;
  a.out_stride = out_image_stride;
  const long long total = static_cast<long long>(n) * c * out_h * out_w;
  return launch(resize_pad_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, cs(stream),
                "resize_pad_kernel", a);
}

int32_t svla_normalize_state(const float* state, int32_t batch, int32_t dim, int32_t ld, const float* p0,
                             const float* p1, int32_t mode, int32_t out_dim, float* out, svla_stream_t stream) {
  if (!state || !p0 || !p1 || !out || batch <= 0 || dim <= 0 || ld < dim || out_dim < dim || (mode != 0 && mode != 1))
    return fail(SVLA_ERR_ARG, "svla_normalize_state: bad args");
  const int total = batch * out_dim;
  return launch(normalize_state_kernel, dim3((total + 255) / 256), dim3(256), 0, cs(stream), "normalize_state_kernel",
                state, batch, dim, ld, p0, p1, mode, out_dim, out);
}

int32_t svla_unnormalize_actions(const float* actions, int32_t rows, int32_t ld, int32_t action_dim, const float* p0,
                                 const float* p1, int32_t mode, float* out, svla_stream_t stream) {
  if (!actions || !p0 || !p1 || !out || rows <= 0 || action_dim <= 0 || ld < action_dim || (mode != 0 && mode != 1))
    return fail(SVLA_ERR_ARG, "svla_unnormalize_actions: bad args");
  const int total = rows * action_dim;
  return launch(unnormalize_actions_kernel, dim3((total + 255) / 256), dim3(256), 0, cs(stream),
                "unnormalize_actions_kernel", actions, rows, ld, action_dim, p0, p1, mode, out);
}

int32_t svla_rope_table(float* c, int32_t max_pos, float max_wavelength, svla_stream_t stream) {
  if (!c || max_pos <= 0 || max_wavelength <= 0.f) return fail(SVLA_ERR_ARG, "svla_rope_table: bad args");
  return launch(rope_table_kernel, dim3((max_pos * 32 + 255) / 256), dim3(256), 0, cs(stream), "rope_table_kernel", reinterpret_cast<float2*>(c), max_pos,
                                                                         max_wavelength);
}

int32_t svla_build_masks(const uint8_t* img_mask0, const uint8_t* img_mask1, const uint8_t* lang_mask, int32_t batch,
                         int32_t n_img, int32_t n_lang, int32_t chunk, uint8_t* prefix_mask, int32_t* prefix_pos,
                         uint8_t* self_mask, uint8_t* cross_mask, int32_t* suffix_pos, int32_t* cross_pos,
                         svla_stream_t stream) {
  if (!img_mask0 || !img_mask1 || !lang_mask || !prefix_mask || !prefix_pos || !self_mask || !cross_mask ||
      !suffix_pos || !cross_pos || batch <= 0 || n_img < 0 || n_lang < 0 || chunk <= 0)
    return fail(SVLA_ERR_ARG, "svla_build_masks: bad args");
  // mask rows are written as 16-byte runs
  if ((reinterpret_cast<uintptr_t>(prefix_mask) | reinterpret_cast<uintptr_t>(self_mask) |
       reinterpret_cast<uintptr_t>(cross_mask)) % 16 != 0)
    return fail(SVLA_ERR_ARG, "svla_build_masks: masks must be 16-byte aligned");
  MaskArgs a{img_mask0, img_mask1, lang_mask, batch, n_img, n_lang, chunk, prefix_mask, prefix_pos,
             self_mask, cross_mask, suffix_pos, cross_pos};
  const int lp = 2 * n_img + n_lang + 1;
  const int rows = lp + 2 * chunk;  // prefix, self-attention and cross-attention mask rows of a sample
  return launch(masks_kernel, dim3(static_cast<unsigned>((rows + 7) / 8), static_cast<unsigned>(batch)), dim3(256), 0,
                cs(stream), "masks_kernel", a);
}

int32_t svla_embed_tokens(const int64_t* tokens, int32_t batch, int32_t t, const void* table, int32_t vocab,
                          int32_t hidden, float scale, void* out, int32_t rows_per_batch, int32_t row_offset,
                          svla_stream_t stream) {
  if (!tokens || !table || !out || batch <= 0 || t <= 0 || vocab <= 0 || hidden <= 0 || hidden % 8)
    return fail(SVLA_ERR_ARG, "svla_embed_tokens: bad args");
  const long long threads = static_cast<long long>(batch) * t * 32;
  return launch(embed_tokens_kernel, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, cs(stream), "embed_tokens_kernel",
                reinterpret_cast<const long long*>(tokens), batch, t, static_cast<const __nv_bfloat16*>(table), vocab, hidden,
      scale, static_cast<__nv_bfloat16*>(out), rows_per_batch, row_offset, device_error_ptr());
}

int32_t svla_im2col(const float* images, int32_t n, int32_t c, int32_t s, int32_t p, void* out, svla_stream_t stream) {
  if (!images || !out || n <= 0 || c <= 0 || p <= 0 || p % 8 || s % p) return fail(SVLA_ERR_ARG, "svla_im2col: bad args");
  const long long total = static_cast<long long>(n) * (s / p) * (s / p) * c * p * (p / 8);
  return launch(im2col_kernel, dim3(static_cast<unsigned>((total + 255) / 256)), dim3(256), 0, cs(stream), "im2col_kernel",
                images, n, c, s, p,
                                                                                     static_cast<__nv_bfloat16*>(out));
}

int32_t svla_f32_to_bf16(const float* x, void* y, int64_t n, svla_stream_t stream) {
  if (!x || !y || n <= 0) return fail(SVLA_ERR_ARG, "svla_f32_to_bf16: bad args");
  return launch(f32_to_bf16_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, cs(stream), "f32_to_bf16_kernel",
                x, static_cast<__nv_bfloat16*>(y), n);
}

int32_t svla_reciprocal(const float* x, float* y, int64_t n, svla_stream_t stream) {
  if (!x || !y || n <= 0) return fail(SVLA_ERR_ARG, "svla_reciprocal: bad args");
  return launch(reciprocal_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, cs(stream), "reciprocal_kernel",
                x, y, n);
}

int32_t svla_euler_init(const float* noise, float* xt, void* xt_bf16, int64_t n, svla_stream_t stream) {
  if (!noise || !xt || !xt_bf16 || n <= 0) return fail(SVLA_ERR_ARG, "svla_euler_init: bad args");
  return launch(euler_init_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0, cs(stream), "euler_init_kernel",
                noise, xt,
                                                                                    static_cast<__nv_bfloat16*>(xt_bf16), n);
}

size_t svla_flow_packed_bytes(int32_t n, int32_t k, int32_t elem_bytes) {
  if (n <= 0 || k <= 0 || n % 16 || k % 16 || (elem_bytes != 1 && elem_bytes != 2)) return 0;
  return static_cast<size_t>(n) * k * elem_bytes;
}

int32_t svla_flow_pack_weight(const void* w, int32_t elem_bytes, int64_t ld, int32_t n, int32_t k, void* out,
                              svla_stream_t stream) {
  if (!w || !out || svla_flow_packed_bytes(n, k, elem_bytes) == 0 || ld < k)
    return fail(SVLA_ERR_ARG, "svla_flow_pack_weight: bad args (n, k multiples of 16, ld >= k, elem_bytes 1 or 2)");
  if (reinterpret_cast<uintptr_t>(out) % 16 != 0 || reinterpret_cast<uintptr_t>(w) % elem_bytes != 0)
    return fail(SVLA_ERR_ARG, "svla_flow_pack_weight: out must be 16-byte aligned");
  const long long total = static_cast<long long>(n) * k / 8;
  const unsigned grid = static_cast<unsigned>(std::min<long long>((total + 255) / 256, 1 << 16));
  return launch(pack_fragments_kernel, dim3(grid), dim3(256), 0, cs(stream), "pack_fragments_kernel",
                static_cast<const uint8_t*>(w), static_cast<int>(elem_bytes), static_cast<long long>(ld),
                static_cast<int>(n), static_cast<int>(k), static_cast<uint8_t*>(out));
}

int32_t svla_flow(const svla_flow_desc* d, svla_stream_t stream) {
  if (!d) return fail(SVLA_ERR_ARG, "svla_flow: null descriptor");
  const int rows = d->batch * d->chunk;
  if (d->batch < 1 || d->chunk < 1 || rows > SVLA_FLOW_MAX_ROWS)
    return fail(SVLA_ERR_ARG, "svla_flow: batch * chunk = %d outside 1..%d", rows, SVLA_FLOW_MAX_ROWS);
  if (d->hidden < 16 || d->hidden % 16 != 0 || d->hidden > kFlowKC)
    return fail(SVLA_ERR_ARG, "svla_flow: hidden %d must be a multiple of 16 in 16..%d", d->hidden, kFlowKC);
  if (d->action_dim < 16 || d->action_dim % 16 != 0 || d->mlp < 16 || d->mlp % 16 != 0)
    return fail(SVLA_ERR_ARG, "svla_flow: action_dim %d and mlp %d must be multiples of 16", d->action_dim, d->mlp);
  if (d->heads < 1 || d->kv_heads < 1 || d->heads % d->kv_heads != 0)
    return fail(SVLA_ERR_ARG, "svla_flow: heads %d not a multiple of kv_heads %d", d->heads, d->kv_heads);
  if (d->n_layers < 1 || d->n_layers > SVLA_FLOW_MAX_LAYERS || d->num_steps < 1 || d->prefix_len < 1)
    return fail(SVLA_ERR_ARG, "svla_flow: n_layers %d (1..%d), num_steps %d, prefix_len %d", d->n_layers,
                SVLA_FLOW_MAX_LAYERS, d->num_steps, d->prefix_len);
  if (d->max_pos < 1) return fail(SVLA_ERR_ARG, "svla_flow: max_pos %d", d->max_pos);
  const void* need[] = {d->noise, d->xt, d->xt_bf16, d->w_action_in, d->b_action_in, d->w_time_in, d->time_in_const,
                        d->w_time_out, d->b_time_out, d->final_norm, d->w_action_out, d->b_action_out, d->suffix_pos,
                        d->cross_pos, d->rope_cs, d->a_emb, d->a_t, d->eh, d->eq, d->ek, d->ev, d->ectx, d->emlp,
                        d->norm_part, d->sync};
  for (const void* p : need)
    if (!p) return fail(SVLA_ERR_ARG, "svla_flow: null pointer argument");
  // 16-byte rows for the staged A loads and the packed stores
  // and the fragment-packed weights (16-byte lane loads)
  const void* aligned[] = {d->xt_bf16, d->a_emb, d->a_t, d->eh, d->eq, d->ek, d->ev, d->ectx, d->emlp, d->rope_cs,
                           d->w_action_in, d->w_time_in, d->w_time_out, d->w_action_out};
  for (const void* p : aligned)
    if (reinterpret_cast<uintptr_t>(p) % 16 != 0) return fail(SVLA_ERR_ARG, "svla_flow: buffers must be 16-byte aligned");
  FlowArgs a{};
  a.B = d->batch; a.S = d->chunk; a.Lp = d->prefix_len; a.E = d->hidden; a.A = d->action_dim;
  a.Hq = d->heads; a.Hkv = d->kv_heads; a.mlp = d->mlp; a.n_layers = d->n_layers; a.n_steps = d->num_steps;
  a.eps = d->eps;
  a.dt = static_cast<float>(-1.0 / d->num_steps);
  a.scale = 0.125f;  // head_dim^-1/2
  a.noise = d->noise; a.xt = d->xt; a.xt_bf = static_cast<__nv_bfloat16*>(d->xt_bf16);
  auto bfp = [](const void* p) { return static_cast<const __nv_bfloat16*>(p); };
  auto u8p = [](const void* p) { return static_cast<const uint8_t*>(p); };
  a.w_in = u8p(d->w_action_in); a.b_in = bfp(d->b_action_in);
  a.w_tin = u8p(d->w_time_in); a.c_step = d->time_in_const;
  a.w_tout = u8p(d->w_time_out); a.b_tout = bfp(d->b_time_out);
  a.ln_f = bfp(d->final_norm); a.w_out = u8p(d->w_action_out); a.b_out = bfp(d->b_action_out);
  a.key_mask = d->key_mask; a.key_mask_bs = d->key_mask_bs;
  a.suffix_pos = d->suffix_pos; a.cross_pos = d->cross_pos; a.rope_cs = d->rope_cs; a.max_pos = d->max_pos;
  auto bfw = [](void* p) { return static_cast<__nv_bfloat16*>(p); };
  a.a_emb = bfw(d->a_emb); a.a_t = bfw(d->a_t); a.eh = bfw(d->eh); a.eq = bfw(d->eq); a.ek = bfw(d->ek);
  a.ev = bfw(d->ev); a.ectx = bfw(d->ectx); a.emlp = bfw(d->emlp); a.norm_part = d->norm_part;
  if (reinterpret_cast<uintptr_t>(d->sync) % 8 != 0) return fail(SVLA_ERR_ARG, "svla_flow: sync must be 8-byte aligned");
  if (d->key_mask && (reinterpret_cast<uintptr_t>(d->key_mask) % 16 != 0 || d->key_mask_bs % 16 != 0 ||
                      d->key_mask_bs < (d->prefix_len + 15) / 16 * 16))
    return fail(SVLA_ERR_ARG, "svla_flow: key flag rows must be 16-byte aligned and hold prefix_len rounded up to 16");
  a.sync = reinterpret_cast<unsigned long long*>(d->sync);
  a.spin_limit = d->spin_limit ? d->spin_limit : kSpinLimit;
  a.dbg = reinterpret_cast<unsigned long long*>(d->debug_clock);
  a.err = device_error_ptr();
  if (!a.err) return fail(SVLA_ERR_CUDA, "svla_flow: device error word unavailable");
  for (int i = 0; i < d->n_layers; ++i) {
    const svla_flow_layer& s = d->layer[i];
    if (!s.input_norm || !s.post_norm || !s.wq || !s.wo || !s.wg || !s.wu || !s.wd || !s.keys || !s.values ||
        !s.sq || !s.so || !s.sg || !s.su || !s.sd || (!s.cross && (!s.wk || !s.wv || !s.sk || !s.sv)))
      return fail(SVLA_ERR_ARG, "svla_flow: layer %d lacks a weight, a weight scale or its keys / values", i);
    const void* packed[] = {s.wq, s.wk, s.wv, s.wo, s.wg, s.wu, s.wd};
    for (const void* p : packed)
      if (reinterpret_cast<uintptr_t>(p) % 16 != 0)
        return fail(SVLA_ERR_ARG, "svla_flow: layer %d: packed weights must be 16-byte aligned", i);
    FlowLayer& L = a.layer[i];
    L.ln1 = bfp(s.input_norm); L.ln2 = bfp(s.post_norm); L.wq = u8p(s.wq); L.wk = u8p(s.wk); L.wv = u8p(s.wv);
    L.wo = u8p(s.wo); L.wg = u8p(s.wg); L.wu = u8p(s.wu); L.wd = u8p(s.wd); L.k1 = bfp(s.keys); L.v1 = bfp(s.values);
    L.sq = s.sq; L.sk = s.sk; L.sv = s.sv; L.so = s.so; L.sg = s.sg; L.su = s.su; L.sd = s.sd;
    L.cross = s.cross ? 1 : 0;
  }
  // one CTA per SM, all resident at once (a cooperative launch refuses a grid that cannot be)
  int dev = 0, sms = 0, per_sm = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return fail(SVLA_ERR_CUDA, "svla_flow: cannot read the SM count");
  const size_t smem = sizeof(FlowSmem);
  static bool configured[64] = {false};  // the attribute is per function and per device
  if (dev < 0 || dev >= 64) return fail(SVLA_ERR_ARG, "device index %d out of range", dev);
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(flow_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "svla_flow: %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, flow_kernel, kFlowThreads, smem) != cudaSuccess ||
      per_sm < 1)
    return fail(SVLA_ERR_CUDA, "svla_flow: the kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms));
  cfg.blockDim = dim3(kFlowThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = cs(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, flow_kernel, a);
  if (e != cudaSuccess) return fail(SVLA_ERR_CUDA, "flow_kernel: %s", cudaGetErrorString(e));
  return check_launch("flow_kernel");
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// SmoothQuant W8A8 linear with built-in scratch, for callers that cannot allocate device memory.
//
// Some callers cannot call cudaMalloc: a robot's fixed-rate control loop that must not allocate
// after start-up (an allocation can block for milliseconds or fail under fragmentation), or a
// foreign-language binding that only holds the device pointers it was handed and has no allocator.
// This entry point takes the same inputs and outputs as svla_sq_linear_w8a8 but no workspace: the
// int8 activations live in one fixed array compiled into the library.
//
// The array is kStaticScratchBytes (4 MiB) of device memory, reserved on every GPU that loads
// the library until the process exits, and shared by every call on that device.  So calls whose
// m * k exceeds 4 MiB are rejected, and calls that overlap on the GPU (two streams, or two
// threads) race on the same bytes and must be serialised by the caller.  Each call overwrites
// every byte it later reads (the quantiser writes all m * k values before the GEMM reads them,
// in stream order), so nothing has to be cleared between calls.
//
// In host code the array's name is only a stand-in symbol, not a device address.  The first call
// on each device asks the runtime for the device address (cudaGetSymbolAddress, with that device
// current) and caches it; that first call should therefore come before any stream capture.
// ------------------------------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;
static __device__ __align__(256) int8_t g_sq_linear_static_scratch[kStaticScratchBytes];

int8_t* static_scratch_address(int32_t* status) {
  static int8_t* addr[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = fail(SVLA_ERR_CUDA, "svla_sq_linear_w8a8_static_scratch: no current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_sq_linear_static_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = fail(SVLA_ERR_CUDA, "svla_sq_linear_w8a8_static_scratch: cudaGetSymbolAddress failed: %s",
                     cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<int8_t*>(p);
  }
  *status = SVLA_OK;
  return addr[dev];
}

}  // namespace

extern "C" int32_t svla_sq_linear_w8a8_static_scratch(const void* x, const float* smooth, float act_scale,
                                                      const int8_t* qweight, const float* wscale, const void* bias,
                                                      int32_t m, int32_t n, int32_t k, void* y,
                                                      svla_stream_t stream) {
  if (m <= 0 || k <= 0 || n <= 0) return fail(SVLA_ERR_ARG, "svla_sq_linear_w8a8_static_scratch: bad shape");
  const size_t need = static_cast<size_t>(m) * static_cast<size_t>(k);
  if (need > kStaticScratchBytes)
    return fail(SVLA_ERR_ARG,
                "svla_sq_linear_w8a8_static_scratch: m*k = %zu bytes of int8 activations exceeds the fixed "
                "scratch of %zu bytes; use svla_sq_linear_w8a8 with a caller-provided workspace",
                need, kStaticScratchBytes);
  int32_t rc = SVLA_OK;
  int8_t* qx = static_scratch_address(&rc);
  if (!qx) return rc;
  rc = svla_quantize_smooth(x, k, smooth, act_scale, qx, k, m, k, stream);
  if (rc) return rc;
  svla_gemm_desc d;
  std::memset(&d, 0, sizeof(d));
  d.kind = SVLA_KIND_I8;
  d.epi = SVLA_EPI_BF16;
  d.m = m;
  d.k = k;
  d.nseg = 1;
  d.seg[0] = svla_gemm_seg{qx, k, qweight, k, wscale, bias, nullptr, y, n, n, act_scale, 0};
  return run_gemm(&d, cs(stream));
}
