// tcgen05 GEMM for sm_100a:  D[M, N] = A[M, K] * B[N, K]^T  (both operands K-major), with fused epilogues.
//
// Operand kinds
//   I8     A int8 (TMA), B int8 (TMA), tcgen05.mma kind::i8 -> int32 in TMEM.   SmoothQuant W8A8 linears.
//   BF16   A bf16 (TMA), B bf16 (TMA), kind::f16 -> fp32 in TMEM.               plain bf16 linears.
//   W8A16  A bf16 (TMA), B int8 (TMA into a staging buffer), converted by the epilogue warps to
//          bf16(q * w_s[n]) in the 128B-swizzled layout the MMA reads, then kind::f16.  W8A16 linears.
//
// CTA pairs (CG = 2): a cluster of two CTAs computes 256-row tiles with tcgen05.mma.cta_group::2 (M = 256);
// each CTA loads its own 128 A rows and half of the tile's B rows, so a k-stage brings 32 KB into each SM
// instead of 48 KB for the same MMA work.  The even CTA issues the MMAs and commits to both CTAs' barriers;
// every load is a plain TMA load of the CTA's own tile.  Opt-in: the main loop is set by the issue rate of
// the MMA thread (about one tcgen05.mma per 170-210 cycles at any N), which the pair form does not change.
//
// Persistent: one CTA (pair) per SM (pair) walks output tiles t = cluster, cluster + clusters, ... in N-fastest
// order (the CTAs running at one time share A row-blocks; the weights stay L2-resident).  Accumulators
// are double-buffered in TMEM (2 x P x BN columns) so the epilogue of one tile overlaps the MMAs of the next.
// Warp roles: warp 0 issues TMA, warp 1 owns TMEM and issues tcgen05.mma (one lane), the next 8 or 16 warps
// run the epilogue (two or four per TMEM lane quarter 32*(warp%4) .. +31, each on its share of the tile's
// columns; see epi_warps), and for W8A16 the last 4 warps convert the int8 weight stages to bf16.  Tile: 128 rows (M) x BN columns (N) x 128
// bytes of K per pipeline stage.
//
// "Segments" let one launch cover several linears that share M and K but have their own A operand,
// weights, scales and outputs (q/k/v with per-projection SmoothQuant activations).  "Pairs" (P = 2)
// compute two accumulators for the same output tile (gate and up) for the SiLU-gate epilogue.
#pragma once

#include "ptx.cuh"

namespace svla {

enum class Kind : int { I8 = 0, BF16 = 1, W8A16 = 2 };

enum class Epi : int {
  Bf16 = 0,       // y = bf16(acc*a*w_s + b) [* post_scale -> bf16]
  I32 = 1,        // raw int32 accumulators
  Rope = 2,       // Bf16, then rotate-half RoPE on segments flagged rope (64-column heads)
  Resid = 3,      // out = bf16(bf16(y) + resid)
  SiluMul = 4,    // pairs: out = bf16(bf16(silu(bf16(g))) * bf16(u))
  GeluQuant = 5,  // g = bf16(gelu_tanh(bf16(y))); optional qout = smooth_quant(g), optional bf16 out
  Euler = 6,      // v = acc + b (fp32); x_t += dt * v; x_t_bf16 = bf16(x_t)
  SiluBf16 = 7,   // out = bf16(silu(bf16(y)))
  F32 = 8,        // out = v in fp32
};

struct GemmSeg {
  const float* wscale;          // [n] per-output-channel weight scale, nullptr means 1
  const __nv_bfloat16* bias;    // [n] or nullptr
  void* out;                    // output base (row 0, column 0 of this segment)
  int ldo;                      // output row stride, elements
  int n;                        // columns in this segment (multiple of 16)
  int tile_begin;               // first blockIdx.y of this segment
  float act_scale;              // activation scale a (I8); 1 otherwise
  int rope;                     // Rope epilogue: rotate this segment
  const float* bias_f32;        // optional fp32 bias [n] added after `bias` (per-step constants)
};

struct GemmArgs {
  CUtensorMap ta[3];
  CUtensorMap tb[3];
  GemmSeg seg[3];
  int nseg;     // segments (P = 1) or 2 for a pair (P = 2)
  int M, K;
  int tiles_m, tiles_n;  // output tiles: ceil(M / 128) x (sum over segments of ceil(n / BN))
  // output row remap: row = (m / rows_per_group) * group_stride + (m % rows_per_group) + row_offset
  int rows_per_group, group_stride, row_offset;
  float post_scale;                 // Bf16: multiply bf16(y) by this and round again (0 = off)
  const __nv_bfloat16* resid;       // Resid: residual rows (may alias out)
  int ldr, resid_rows;              // resid row = (resid_rows > 0 ? m % resid_rows : remapped row)
  const float2* rope_cs;            // [max_pos][32] (cos, sin)
  const int* pos;                   // [M] positions
  int max_pos;
  const float* q_smooth;            // GeluQuant: smooth vector of the next linear [N]
  const float* q_rsmooth;           // GeluQuant: optional 1 / q_smooth
  float q_act;                      // GeluQuant: activation scale of the next linear
  int8_t* qout;                     // GeluQuant: int8 output [M, ldq]
  int ldq;
  float dt;                         // Euler
  float* xt;                        // Euler: fp32 state [M, ldo]
  __nv_bfloat16* xt_bf16;           // Euler: bf16 copy
  unsigned long long* dbg;          // optional phase clock stamps of CTA 0 (profiling)
  int weights_resident;             // B operands were written before the previous kernel started
  int shared_a;                     // pair over one A operand (P = 2, single CTAs): A is loaded once per
                                    // stage and each k-step is ONE MMA of N = 2 * BN over the adjacent B tiles
  int out_v8;                       // every bf16 output row start is 32-byte aligned: 256-bit stores
  int resid_v8;                     // every residual row start is 32-byte aligned: 256-bit loads
  // split-K: work item t is split t % splits (k-tiles [split * kt_per_split, +kt_per_split)) of output
  // tile t / splits.  Every split stores its raw 32-bit accumulators to `partial`; the last to arrive on
  // the tile's counter adds them in split order into its own accumulator and runs the epilogue.
  int splits, kt_per_split;
  uint32_t* partial;                // [tiles][splits][P][128][BN]
  int* counters;                    // [tiles], zero between launches (the last split resets it)
  int* err;
};

__device__ __forceinline__ void stamp(unsigned long long* dbg, int slot) {
  if (dbg != nullptr && blockIdx.x == 0) dbg[slot] = clock64();
}

template <Kind KIND>
struct KindTraits;
template <>
struct KindTraits<Kind::I8> {
  static constexpr int kBK = 128;  // K elements per stage (128 bytes)
  static constexpr int kKStep = 32;  // K per MMA instruction
  static constexpr bool kConvert = false;
  static __device__ __forceinline__ uint32_t idesc(int n) { return idesc_i8(128, n); }
};
template <>
struct KindTraits<Kind::BF16> {
  static constexpr int kBK = 64;
  static constexpr int kKStep = 16;
  static constexpr bool kConvert = false;
  static __device__ __forceinline__ uint32_t idesc(int n) { return idesc_bf16(128, n); }
};
template <>
struct KindTraits<Kind::W8A16> {
  static constexpr int kBK = 64;
  static constexpr int kKStep = 16;
  static constexpr bool kConvert = true;
  static __device__ __forceinline__ uint32_t idesc(int n) { return idesc_bf16(128, n); }
};

template <Kind KIND, int BN, int P, int STAGES, int CG = 1>
struct GemmSmem {
  static constexpr int kATile = 128 * 128;            // bytes
  static constexpr int kBTile = (BN / CG) * 128;      // bytes (bf16 or int8 MMA operand; a CTA pair splits B)
  static constexpr int kRawTile = KindTraits<KIND>::kConvert ? BN * 64 : 0;  // int8 staging, W8A16
  static constexpr int kStage = P * (kATile + kBTile + kRawTile);
  static constexpr int kBarOff = STAGES * kStage;
  // per-tile column constants staged by the epilogue warps: 2 buffers x kConstArrays x BN floats
  static constexpr int kConstArrays = 6;  // scale0, bias0, scale1, bias1, next-linear smooth, its reciprocal
  static constexpr int kConstOff = kBarOff + 256;
  static constexpr int kBytes = kConstOff + 2 * kConstArrays * BN * 4 + 1024;  // + alignment slack
  static constexpr int kAccCols = P * BN;              // one accumulator buffer
  static constexpr int kTmemCols = (2 * kAccCols <= 32) ? 32 : (2 * kAccCols <= 64) ? 64 : (2 * kAccCols <= 128) ? 128
                                   : (2 * kAccCols <= 256) ? 256 : 512;
  static_assert(2 * kAccCols <= 512, "two accumulator buffers must fit in TMEM");
  static_assert(kBytes <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
};

// Epilogue warps: 16 (four per TMEM lane quarter, each on a quarter of the tile's columns) for the GELU +
// SmoothQuant epilogue, whose long per-element arithmetic chain needs the extra warps to hide its latency
// (measured 884 -> 638 us on the SigLIP fc1); 8 (two per lane quarter, half the columns each) for the
// others, which are bound by their row-wise stores and gain nothing from more warps but register pressure.
template <Kind KIND, int P, Epi EPI>
__host__ __device__ constexpr int epi_warps() { return (EPI == Epi::GeluQuant && P == 1 && !KindTraits<KIND>::kConvert) ? 16 : 8; }

template <Kind KIND, int P, Epi EPI>
__host__ __device__ constexpr int gemm_threads() { return 32 * (2 + epi_warps<KIND, P, EPI>() + (KindTraits<KIND>::kConvert ? 4 : 0)); }

// SiLU x * sigmoid(x) and tanh-GELU 0.5 x (1 + tanh(u)) = x * sigmoid(2u), u = sqrt(2/pi)(x + 0.044715 x^3),
// both evaluated as x / (1 + 2^(-z log2 e)) with the hardware 2^x and reciprocal approximations: the results
// are rounded to bf16 (8 significant bits) right after, far coarser than these (about 2^-20 relative).
// For x -> -inf the exponential overflows to +inf and the quotient goes to -0, the limit of both.
__device__ __forceinline__ float silu_f(float x) {
  return __fmul_rn(x, rcp_approx(__fadd_rn(1.0f, ex2_approx(__fmul_rn(x, -1.4426950408889634f)))));
}
__device__ __forceinline__ float gelu_tanh_f(float x) {
  // -2 u log2(e) = x (c0 + c1 x^2), c0 = -2 sqrt(2/pi) log2(e), c1 = 0.044715 c0
  constexpr float c0 = -2.302208198f, c1 = -0.1029432396f;
  const float z = __fmul_rn(x, __fmaf_rn(c1, __fmul_rn(x, x), c0));
  return __fmul_rn(x, rcp_approx(__fadd_rn(1.0f, ex2_approx(z))));
}
// Two lanes of silu_f / gelu_tanh_f through the packed fp32 pipe: every packed lane rounds exactly as the
// scalar op it replaces, so the results are bit-identical to the scalar forms above.
__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }
__device__ __forceinline__ float2 silu_f2(float2 x) {
  const float2 z = __fmul2_rn(x, f2(-1.4426950408889634f));
  const float2 d = __fadd2_rn(f2(1.0f), make_float2(ex2_approx(z.x), ex2_approx(z.y)));
  return __fmul2_rn(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}
__device__ __forceinline__ float2 gelu_tanh_f2(float2 x) {
  constexpr float c0 = -2.302208198f, c1 = -0.1029432396f;
  const float2 z = __fmul2_rn(x, __ffma2_rn(f2(c1), __fmul2_rn(x, x), f2(c0)));
  const float2 d = __fadd2_rn(f2(1.0f), make_float2(ex2_approx(z.x), ex2_approx(z.y)));
  return __fmul2_rn(x, make_float2(rcp_approx(d.x), rcp_approx(d.y)));
}

template <int BN, int P, int CG = 1>
__device__ __forceinline__ void tile_coord(const GemmArgs& a, int t, int& si, int& m0, int& n0, int rank = 0) {
  if (a.splits > 1) t /= a.splits;
  const int nt = t % a.tiles_n, mt = t / a.tiles_n;
  si = 0;
  if constexpr (P == 1) {
#pragma unroll
    for (int s = 1; s < 3; ++s)
      if (s < a.nseg && nt >= a.seg[s].tile_begin) si = s;
  }
  m0 = mt * 128 * CG + rank * 128;
  n0 = (nt - a.seg[si].tile_begin) * BN;
}

// k-tile range [kb, ke) of work item t
__device__ __forceinline__ void k_range(const GemmArgs& a, int t, int k_tiles, int& kb, int& ke) {
  if (a.splits > 1) {
    kb = (t % a.splits) * a.kt_per_split;
    ke = kb + a.kt_per_split < k_tiles ? kb + a.kt_per_split : k_tiles;
  } else {
    kb = 0;
    ke = k_tiles;
  }
}

// Epilogue of one output tile for the calling warp's 32 TMEM lanes (rows row = 32*(warp%4) + lane) and
// its share of the columns (kEpiParts warps share each lane quarter).  `ok` is warp-uniform; when false the
// TMEM loads are skipped and nothing is written.
template <Kind KIND, int BN, int P, Epi EPI, int kEpiParts, typename WaitAcc>
__device__ __forceinline__ bool epilogue_tile(const GemmArgs& args, int si, int m0, int n0, uint32_t t_row,
                                              int row, int part, bool ok_in, const float* consts, WaitAcc&& wait_acc) {
  const GemmSeg& sg = args.seg[si];
  const int m = m0 + row;
  bool ok = ok_in;
  bool row_ok = ok && (m < args.M);
  int orow = m;
  if (args.rows_per_group > 0) orow = (m / args.rows_per_group) * args.group_stride + (m % args.rows_per_group);
  orow += args.row_offset;

  // per-column constants of 16 columns starting at nb (staged in shared memory for this tile): set 0
  // belongs to the tile's segment, set 1 to the second linear of a pair.  A missing weight scale is staged
  // as 1 and a missing bias as -0, so both apply unconditionally as exact no-ops.
  auto col_consts = [&](int set, int nb, float (&sc)[16], float (&bi)[16]) {
    const float* scs = consts + (2 * set) * BN + (nb - n0);
    const float* bis = consts + (2 * set + 1) * BN + (nb - n0);
#pragma unroll
    for (int j = 0; j < 16; j += 4) {
      const float4 w = *reinterpret_cast<const float4*>(scs + j);
      const float4 b = *reinterpret_cast<const float4*>(bis + j);
      sc[j] = w.x; sc[j + 1] = w.y; sc[j + 2] = w.z; sc[j + 3] = w.w;
      bi[j] = b.x; bi[j + 1] = b.y; bi[j + 2] = b.z; bi[j + 3] = b.w;
    }
  };
  // v = ((acc * a) * w_s + b_bf16) [+ b_f32]   (I8),   acc + b_bf16 [+ b_f32] otherwise; 16 columns.
  auto dequant16 = [&](const GemmSeg& g, int set, const uint32_t* raw, int nb, float (&v)[16]) {
    float sc[16], bi[16];
    col_consts(set, nb, sc, bi);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      float2 x;
      if constexpr (KIND == Kind::I8)
        x = __fmul2_rn(__fmul2_rn(make_float2(static_cast<float>(static_cast<int>(raw[j])),
                                              static_cast<float>(static_cast<int>(raw[j + 1]))),
                                  f2(g.act_scale)),
                       make_float2(sc[j], sc[j + 1]));
      else
        x = make_float2(__uint_as_float(raw[j]), __uint_as_float(raw[j + 1]));
      const float2 y = __fadd2_rn(x, make_float2(bi[j], bi[j + 1]));
      v[j] = y.x;
      v[j + 1] = y.y;
    }
    if (g.bias_f32 != nullptr) {
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const float2 y = __fadd2_rn(make_float2(v[j], v[j + 1]), make_float2(g.bias_f32[nb + j], g.bias_f32[nb + j + 1]));
        v[j] = y.x;
        v[j + 1] = y.y;
      }
    }
  };
  auto round16 = [](float (&v)[16]) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) bf16_round2(v[j], v[j + 1]);
  };
  auto map2 = [](float (&v)[16], auto fn) {
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 y = fn(make_float2(v[j], v[j + 1]));
      v[j] = y.x;
      v[j + 1] = y.y;
    }
  };
  // 16 bf16 (32 bytes) of one row: one 256-bit store when the outputs allow it (each thread writes its own
  // row, so a warp's store touches 32 rows: half as many store instructions halve the L1 work), else two
  // 128-bit stores
  const bool out_v8 = args.out_v8 != 0;
  auto store_bf16_16 = [out_v8](__nv_bfloat16* o, const float (&v)[16]) {
    uint32_t pk[8];
#pragma unroll
    for (int q2 = 0; q2 < 8; ++q2) pk[q2] = pack_bf16_rn(v[2 * q2], v[2 * q2 + 1]);
    if (out_v8) {
      asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(o), "r"(pk[0]), "r"(pk[1]),
                   "r"(pk[2]), "r"(pk[3]), "r"(pk[4]), "r"(pk[5]), "r"(pk[6]), "r"(pk[7])
                   : "memory");
    } else {
      *reinterpret_cast<int4*>(o) = make_int4(pk[0], pk[1], pk[2], pk[3]);
      *reinterpret_cast<int4*>(o + 8) = make_int4(pk[4], pk[5], pk[6], pk[7]);
    }
  };

  if constexpr (EPI == Epi::Rope) {
    ok = ok && wait_acc();
    row_ok = ok && (m < args.M);
    // one 64-column head at a time (the two warps of a lane quarter take alternate heads), rotated in two
    // blocks of 16 pairs (columns j..j+15 with j+32..j+47) to bound register use
    for (int c = part * 64; c < BN; c += 64 * kEpiParts) {  // kEpiParts warps take alternate heads
      const int nb = n0 + c;
      const bool do_head = row_ok && nb < sg.n;
      int p = 0;
      if (do_head && sg.rope) {
        p = args.pos[m];
        p = p < 0 ? 0 : (p >= args.max_pos ? args.max_pos - 1 : p);
      }
      const float4* cs = reinterpret_cast<const float4*>(args.rope_cs + static_cast<size_t>(p) * 32);
#pragma unroll
      for (int blk = 0; blk < 2; ++blk) {
        const int j0 = blk * 16;
        uint32_t r1[16], r2[16];
        if (ok) {
          tmem_ld16(t_row + c + j0, r1);
          tmem_ld16(t_row + c + j0 + 32, r2);
          tmem_ld_wait();
        }

        if (!do_head) continue;
        float v1[16], v2[16];
        dequant16(sg, 0, r1, nb + j0, v1);
        dequant16(sg, 0, r2, nb + j0 + 32, v2);
        round16(v1);
        round16(v2);
        if (sg.rope) {
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float4 t = cs[(j0 + j) / 2];  // (cos_i, sin_i, cos_i+1, sin_i+1), i = j0 + j
            float x1 = v1[j], x2 = v2[j];
            v1[j] = __fsub_rn(__fmul_rn(x1, t.x), __fmul_rn(x2, t.y));
            v2[j] = __fadd_rn(__fmul_rn(x2, t.x), __fmul_rn(x1, t.y));
            x1 = v1[j + 1];
            x2 = v2[j + 1];
            v1[j + 1] = __fsub_rn(__fmul_rn(x1, t.z), __fmul_rn(x2, t.w));
            v2[j + 1] = __fadd_rn(__fmul_rn(x2, t.z), __fmul_rn(x1, t.w));
          }
        }
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb + j0;
        store_bf16_16(o, v1);
        store_bf16_16(o + 32, v2);
      }
    }
  } else {
    constexpr int kPart = BN / kEpiParts;          // columns of this warp
    constexpr int kChunk = kPart >= 32 ? 32 : 16;  // columns per TMEM round trip
    constexpr int kNC = kPart / kChunk;            // chunks per warp and tile
    constexpr int kRes = (EPI == Epi::Resid) ? kChunk / 8 : 1;
    const float ra = (EPI == Epi::GeluQuant && args.qout) ? __frcp_rn(args.q_act) : 0.0f;
    const int c0 = part * kPart;
    const int rrow = (EPI == Epi::Resid && args.resid_rows > 0) ? (m % args.resid_rows) : orow;
    // residual rows do not depend on the accumulator: fetch them ahead of it
    auto load_res = [&](int4 (&res)[kRes], int cb) {
      if constexpr (EPI == Epi::Resid) {
        const bool in = ok && m < args.M;
        const __nv_bfloat16* rs = args.resid + static_cast<size_t>(rrow) * args.ldr + n0 + cb;
        // 16 columns (32 bytes) per load: one 256-bit load when the residual rows allow it (segment widths
        // are multiples of 16, so both halves of a 16-column group are inside or outside together)
#pragma unroll
        for (int u = 0; u < kRes; u += 2) {
          const bool col_in = in && n0 + cb + u * 8 < sg.n;
          if (col_in && args.resid_v8) {
            uint32_t w[8];
            asm volatile("ld.global.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                         : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
                         : "l"(rs + u * 8)
                         : "memory");
            res[u] = make_int4(w[0], w[1], w[2], w[3]);
            res[u + 1] = make_int4(w[4], w[5], w[6], w[7]);
          } else {
            res[u] = col_in ? *reinterpret_cast<const int4*>(rs + u * 8) : make_int4(0, 0, 0, 0);
            res[u + 1] = col_in ? *reinterpret_cast<const int4*>(rs + u * 8 + 8) : make_int4(0, 0, 0, 0);
          }
        }
      }
    };
    auto tmem_load = [&](uint32_t (&r)[kChunk], uint32_t (&r2)[P == 2 ? kChunk : 1], int cb) {
      if (ok) {
#pragma unroll
        for (int u = 0; u < kChunk; u += 16) {
          tmem_ld16(t_row + cb + u, *reinterpret_cast<uint32_t(*)[16]>(&r[u]));
          if constexpr (P == 2) tmem_ld16(t_row + BN + cb + u, *reinterpret_cast<uint32_t(*)[16]>(&r2[u]));
        }
      }
    };
    auto process = [&](const uint32_t (&r)[kChunk], const uint32_t (&r2)[P == 2 ? kChunk : 1], const int4 (&res)[kRes],
                       int cb) {
#pragma unroll
      for (int u = 0; u < kChunk; u += 16) {
        const int nb = n0 + cb + u;
        if (!row_ok || nb >= sg.n) continue;
        const uint32_t* rr = &r[u];
        if constexpr (EPI == Epi::I32) {
          int* o = reinterpret_cast<int*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb;
#pragma unroll
          for (int j = 0; j < 16; j += 4) *reinterpret_cast<int4*>(o + j) = make_int4(rr[j], rr[j + 1], rr[j + 2], rr[j + 3]);
          continue;
        }
        float v[16];
        dequant16(sg, 0, rr, nb, v);
        if constexpr (EPI == Epi::F32) {
          float* o = reinterpret_cast<float*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb;
#pragma unroll
          for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else if constexpr (EPI == Epi::Euler) {
          float* xo = args.xt + static_cast<size_t>(orow) * sg.ldo + nb;
          __nv_bfloat16* xb = args.xt_bf16 + static_cast<size_t>(orow) * sg.ldo + nb;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float x = __fadd_rn(xo[j], __fmul_rn(args.dt, v[j]));
            xo[j] = x;
            xb[j] = __float2bfloat16_rn(x);
          }
        } else {
          if constexpr (EPI == Epi::SiluMul) {
            float uv[16];
            dequant16(args.seg[1], 1, &r2[u], nb, uv);
            round16(v);
            round16(uv);
            map2(v, [](float2 x) { return silu_f2(x); });
            round16(v);
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
              const float2 y = __fmul2_rn(make_float2(v[j], v[j + 1]), make_float2(uv[j], uv[j + 1]));
              v[j] = y.x;
              v[j + 1] = y.y;
            }
          } else if constexpr (EPI == Epi::SiluBf16) {
            round16(v);
            map2(v, [](float2 x) { return silu_f2(x); });
          } else if constexpr (EPI == Epi::Resid) {
            round16(v);
            const int4 ra4 = res[u / 8], rb4 = res[u / 8 + 1];
            const uint32_t rw[8] = {static_cast<uint32_t>(ra4.x), static_cast<uint32_t>(ra4.y),
                                    static_cast<uint32_t>(ra4.z), static_cast<uint32_t>(ra4.w),
                                    static_cast<uint32_t>(rb4.x), static_cast<uint32_t>(rb4.y),
                                    static_cast<uint32_t>(rb4.z), static_cast<uint32_t>(rb4.w)};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float2 y = __fadd2_rn(make_float2(v[2 * j], v[2 * j + 1]),
                                          make_float2(__uint_as_float(rw[j] << 16), __uint_as_float(rw[j] & 0xFFFF0000u)));
              v[2 * j] = y.x;
              v[2 * j + 1] = y.y;
            }
          } else if constexpr (EPI == Epi::GeluQuant) {
            round16(v);
            map2(v, [](float2 x) { return gelu_tanh_f2(x); });
            round16(v);
            if (args.qout != nullptr) {
              uint32_t w[4] = {0u, 0u, 0u, 0u};
              uint32_t slow = 0xFFFFu;  // every element exact when there is no reciprocal smooth vector
              if (args.q_rsmooth != nullptr) {
                slow = 0u;
                const float* rsc = consts + 5 * BN + (nb - n0);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                  w[k] = smooth_quant4_fast(&v[4 * k], *reinterpret_cast<const float4*>(rsc + 4 * k), ra, slow, 4 * k);
              }
              if (slow != 0u) {  // rare: values near a rounding boundary take the two-divide path one by one
                const float* smc = consts + 4 * BN + (nb - n0);
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                  if (slow & (1u << e)) {
                    const uint32_t q8 = static_cast<uint32_t>(smooth_quant_slow(v[e], smc[e], args.q_act) & 0xFF);
                    w[e / 4] = (w[e / 4] & ~(0xFFu << (8 * (e % 4)))) | (q8 << (8 * (e % 4)));
                  }
                }
              }
              *reinterpret_cast<int4*>(args.qout + static_cast<size_t>(orow) * args.ldq + nb) = make_int4(w[0], w[1], w[2], w[3]);
            }
            if (sg.out == nullptr) continue;
          } else if constexpr (EPI == Epi::Bf16) {
            if (args.post_scale != 0.0f) {
              round16(v);
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(v[j], args.post_scale);
            }
          }
          store_bf16_16(reinterpret_cast<__nv_bfloat16*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb, v);
        }
      }
    };
    // tcgen05.ld writes its registers asynchronously until tcgen05.wait::ld, so each chunk's TMEM load is
    // waited for before any other register work; the residual (an ordinary load) of the next chunk is
    // requested before that wait so its latency overlaps it.
    uint32_t r[kChunk], r2[P == 2 ? kChunk : 1];
    int4 resA[kRes], resB[kRes];
    load_res(resA, c0);
    ok = ok && wait_acc();
    row_ok = ok && (m < args.M);
#pragma unroll 1
    for (int i = 0; i < kNC; i += 2) {
      tmem_load(r, r2, c0 + i * kChunk);
      if (i + 1 < kNC) load_res(resB, c0 + (i + 1) * kChunk);
      if (ok) tmem_ld_wait();
      process(r, r2, resA, c0 + i * kChunk);
      if (i + 1 < kNC) {
        tmem_load(r, r2, c0 + (i + 1) * kChunk);
        if (i + 2 < kNC) load_res(resA, c0 + (i + 2) * kChunk);
        if (ok) tmem_ld_wait();
        process(r, r2, resB, c0 + (i + 1) * kChunk);
      }
    }
  }
  return ok;
}

// Split-K step of one output tile, run by all epilogue warps (each on its TMEM lane quarter and share of
// the columns): store this split's raw accumulators; count the arrival; the tile's last split adds all
// partials in split order (int32 exactly, fp32 in a fixed order) into its own accumulator.  Returns
// whether this CTA runs the tile's epilogue.
template <Kind KIND, int BN, int P, int kEpiParts, typename WaitAcc>
__device__ __forceinline__ bool splitk_reduce(const GemmArgs& args, int t, int m0, int row, int part, int etid,
                                              uint32_t t_row, bool ok, volatile int* split_last, WaitAcc&& wait_acc) {
  constexpr int kEpiThreads = 32 * 4 * kEpiParts;
  const int tile = t / args.splits, sp = t % args.splits;
  const bool aok = ok && wait_acc();
  const bool row_in = m0 + row < args.M;
  uint32_t* tile_part = args.partial + static_cast<size_t>(tile) * args.splits * (P * 128 * BN);
#pragma unroll
  for (int p = 0; p < P; ++p) {
#pragma unroll
    for (int c = part * (BN / kEpiParts); c < (part + 1) * (BN / kEpiParts); c += 16) {
      uint32_t r[16];
      if (aok) {
        tmem_ld16(t_row + p * BN + c, r);
        tmem_ld_wait();
      }
      if (aok && row_in) {
        uint32_t* dst = tile_part + (static_cast<size_t>(sp) * P + p) * (128 * BN) + row * BN + c;
#pragma unroll
        for (int u = 0; u < 16; u += 4) *reinterpret_cast<int4*>(dst + u) = make_int4(r[u], r[u + 1], r[u + 2], r[u + 3]);
      }
    }
  }
  // The CTA barrier orders every warp's partial stores before thread 0's gpu-scope release fence (fences
  // are cumulative), which orders them before its counter increment; its acquire fence after the
  // increment orders the other splits' stores before this CTA's reads.
  if (etid == 0 && t == static_cast<int>(blockIdx.x)) stamp(args.dbg, 11);
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
  if (etid == 0 && t == static_cast<int>(blockIdx.x)) stamp(args.dbg, 12);
  if (etid == 0) {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
    *split_last = (atomicAdd(&args.counters[tile], 1) == args.splits - 1) ? 1 : 0;
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
  }
  if (etid == 0 && t == static_cast<int>(blockIdx.x)) stamp(args.dbg, 13);
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
  if (etid == 0 && t == static_cast<int>(blockIdx.x)) stamp(args.dbg, *split_last ? 14 : 15);
  if (*split_last == 0) return false;
#pragma unroll
  for (int p = 0; p < P; ++p) {
#pragma unroll
    for (int c = part * (BN / kEpiParts); c < (part + 1) * (BN / kEpiParts); c += 16) {
      uint32_t acc[16];
#pragma unroll
      for (int u = 0; u < 16; ++u) acc[u] = 0u;
      if (aok && row_in) {
        // eight columns at a time with four splits' loads in flight, added in split order
#pragma unroll
        for (int h8 = 0; h8 < 16; h8 += 8) {
          for (int k0 = 0; k0 < args.splits; k0 += 4) {
            int4 v[4][2];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              if (k0 + kk < args.splits) {
                const uint32_t* src = tile_part + (static_cast<size_t>(k0 + kk) * P + p) * (128 * BN) + row * BN + c + h8;
                v[kk][0] = __ldcg(reinterpret_cast<const int4*>(src));
                v[kk][1] = __ldcg(reinterpret_cast<const int4*>(src + 4));
              }
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              if (k0 + kk < args.splits) {
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  const uint32_t w[4] = {static_cast<uint32_t>(v[kk][u].x), static_cast<uint32_t>(v[kk][u].y),
                                         static_cast<uint32_t>(v[kk][u].z), static_cast<uint32_t>(v[kk][u].w)};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    uint32_t& a = acc[h8 + 4 * u + e];
                    if (k0 + kk == 0)
                      a = w[e];
                    else if constexpr (KIND == Kind::I8)
                      a = static_cast<uint32_t>(static_cast<int>(a) + static_cast<int>(w[e]));
                    else
                      a = __float_as_uint(__fadd_rn(__uint_as_float(a), __uint_as_float(w[e])));
                  }
                }
              }
            }
          }
        }
      }
      if (aok) tmem_st16(t_row + p * BN + c, acc);
    }
  }
  tmem_st_wait();
  // the epilogue may read columns another warp of this lane quarter summed (RoPE takes whole heads)
  tc_fence_before();
  asm volatile("bar.sync 1, %0;" ::"n"(kEpiThreads) : "memory");
  tc_fence_after();
  if (etid == 0) args.counters[tile] = 0;  // ready for the next launch
  return true;
}

template <Kind KIND, int BN, int P, int STAGES, Epi EPI, int CG>
__global__ void __launch_bounds__(gemm_threads<KIND, P, EPI>(), 1) gemm_sm100_kernel(const __grid_constant__ GemmArgs args) {
  constexpr int kEpiWarps = epi_warps<KIND, P, EPI>();
  using T = KindTraits<KIND>;
  using S = GemmSmem<KIND, BN, P, STAGES, CG>;
  static_assert(CG == 1 || (!T::kConvert && BN >= 128), "CTA pairs: I8 / BF16 operands, 128- or 256-column tiles");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;          // W8A16: converted B ready
  uint64_t* tfull = conv + STAGES;          // [2] accumulator buffer holds a finished tile
  uint64_t* tempty = tfull + 2;             // [2] epilogue has drained the accumulator buffer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* split_last = abort_flag + 1;  // split-K: this CTA was the tile's last split

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int k_tiles = (args.K + T::kBK - 1) / T::kBK;
  const int n_tiles_total = args.tiles_m * args.tiles_n * (args.splits > 1 ? args.splits : 1);
  // work units: tiles of 128 * CG rows, walked by clusters (single CTAs when CG = 1)
  const uint32_t rank = (CG == 2) ? cluster_ctarank() : 0u;
  const int cl = blockIdx.x / CG, n_cl = gridDim.x / CG;
  const bool leader = rank == 0;
  // the leader's copy of a barrier (cluster address); the MMA issuer and its commits use these
  auto leader_bar = [&](uint64_t* bar) -> uint32_t { return CG == 2 ? mapa_shared(smem_u32(bar), 0) : smem_u32(bar); };

  if (threadIdx.x == 0) stamp(args.dbg, 0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 4);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], CG * kEpiWarps);  // a pair: the leader's counts both CTAs' epilogue warps
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, S::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, S::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (CG == 2) cluster_sync();  // both CTAs' barriers are initialised before either uses the other's
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (threadIdx.x == 0) stamp(args.dbg, 1);

  auto bounded_wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
      if (mbar_try_wait(bar, parity)) return true;
      if ((i & 1023) == 1023 && *abort_flag) return false;
    }
    record_error(args.err, kErrMbarTimeout);
    *abort_flag = 1;
    return false;
  };
  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      for (int p = 0; p < (P == 1 ? args.nseg : 2); ++p) {
        prefetch_tmap(&args.ta[p]);
        prefetch_tmap(&args.tb[p]);
      }
      constexpr uint32_t kBBytes = T::kConvert ? S::kRawTile : S::kBTile;
      constexpr uint32_t kStageTx = CG * P * (S::kATile + kBBytes);  // bytes both CTAs of the unit bring in
      const bool one_a = P == 2 && args.shared_a;                        // the pair's A tile is loaded once
      const uint32_t stage_tx = kStageTx - (one_a ? static_cast<uint32_t>(CG * S::kATile) : 0u);
      auto b_dst = [&](uint8_t* st, int p) {
        return T::kConvert ? st + P * (S::kATile + S::kBTile) + p * S::kRawTile : st + P * S::kATile + p * S::kBTile;
      };
      // a load of this CTA's tile that completes on the leader's full barrier of stage s
      auto load = [&](void* dst, const CUtensorMap* map, int s, int x, int y) {
        if constexpr (CG == 2)
          tma_load_2d_pair(dst, map, leader_bar(&full[s]), x, y);
        else
          tma_load_2d(dst, map, &full[s], x, y);
      };
      const int b_row0 = static_cast<int>(rank) * (BN / CG);  // a pair: this CTA's half of the B rows
      // Weights packed before the previous kernel started (weights_resident) do not depend on it: the first
      // tile's first STAGES weight tiles are requested before waiting, so they stream in while it finishes.
      int pre = 0;
      if (args.weights_resident && cl < n_tiles_total) {
        int si, m0, n0, kb, ke;
        tile_coord<BN, P, CG>(args, cl, si, m0, n0, rank);
        k_range(args, cl, k_tiles, kb, ke);
        pre = ke - kb < STAGES ? ke - kb : STAGES;
        for (int i = 0; i < pre; ++i) {
          uint8_t* st = smem + i * S::kStage;
          if (leader) mbar_arrive_expect_tx(&full[i], stage_tx);
#pragma unroll
          for (int p = 0; p < P; ++p)
            load(b_dst(st, p), &args.tb[(P == 1) ? si : p], i, (kb + i) * T::kBK, n0 + b_row0);
        }
      }
      pdl_wait();
      pdl_trigger();
      uint32_t g = 0;
      bool ok = true;
      for (int t = cl; t < n_tiles_total && ok; t += n_cl) {
        int si, m0, n0, kb, ke;
        tile_coord<BN, P, CG>(args, t, si, m0, n0, rank);
        k_range(args, t, k_tiles, kb, ke);
        for (int kt = kb; kt < ke; ++kt, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          uint8_t* st = smem + s * S::kStage;
          if (static_cast<int>(g) < pre) {  // weights already requested: only the activations remain
#pragma unroll
            for (int p = 0; p < (one_a ? 1 : P); ++p) load(st + p * S::kATile, &args.ta[(P == 1) ? si : p], s, kt * T::kBK, m0);
            if (g == 0) stamp(args.dbg, 2);
            continue;
          }
          if (!(ok = bounded_wait(&empty[s], ph ^ 1))) break;
          if (leader) mbar_arrive_expect_tx(&full[s], stage_tx);
#pragma unroll
          for (int p = 0; p < P; ++p) {
            const int mi = (P == 1) ? si : p;
            if (p == 0 || !one_a) load(st + p * S::kATile, &args.ta[mi], s, kt * T::kBK, m0);
            load(b_dst(st, p), &args.tb[mi], s, kt * T::kBK, n0 + b_row0);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (a pair: the leader only, for both CTAs)
    if (lane == 0 && leader) {
      // M = 128 per CTA, 256 for a pair
      const uint32_t idesc = (KIND == Kind::I8) ? idesc_i8(128 * CG, BN) : idesc_bf16(128 * CG, BN);
      // a commit to the barrier `bar` of both CTAs of the unit
      auto commit = [&](uint64_t* bar) {
        if constexpr (CG == 2) {
          mma_commit_pair(mapa_shared(smem_u32(bar), 0));
          mma_commit_pair(mapa_shared(smem_u32(bar), 1));
        } else {
          mma_commit(bar);
        }
      };
      uint32_t g = 0, lt = 0;
      bool ok = true;
      for (int t = cl; t < n_tiles_total && ok; t += n_cl, ++lt) {
        const uint32_t ab = lt & 1, use = lt >> 1;
        if (lt < 8) stamp(args.dbg, 16 + 2 * lt);  // profiling: waits here mean the epilogue sets the pace
        if (!(ok = bounded_wait(&tempty[ab], (use & 1) ^ 1))) break;
        if (lt < 8) stamp(args.dbg, 17 + 2 * lt);
        tc_fence_after();
        const uint32_t d_base = tmem_base + ab * S::kAccCols;
        int kb, ke;
        k_range(args, t, k_tiles, kb, ke);
        for (int kt = kb; kt < ke; ++kt, ++g) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          ok = bounded_wait(&full[s], ph);
          if (g == 0) stamp(args.dbg, 3);
          if (ok && T::kConvert) ok = bounded_wait(&conv[s], ph);
          if (g == 0) stamp(args.dbg, 4);
          if (!ok) break;
          tc_fence_after();
          uint8_t* st = smem + s * S::kStage;
          if constexpr (P == 2 && CG == 1 && 2 * BN <= 256) {
            if (args.shared_a) {
              // gate and up over the same A: their B tiles are adjacent in the stage (BN rows each), so one
              // MMA of N = 2 * BN writes both accumulators (columns [0, BN) and [BN, 2 * BN) of the buffer)
              // with half the MMA instructions
              const uint32_t a_addr = smem_u32(st);
              const uint32_t b_addr = smem_u32(st + P * S::kATile);
              const uint32_t idesc2 = T::idesc(2 * BN);
#pragma unroll
              for (int kk = 0; kk < 128 / 32; ++kk) {
                const uint64_t ad = smem_desc_sw128(a_addr + kk * 32);
                const uint64_t bd = smem_desc_sw128(b_addr + kk * 32);
                const uint32_t acc = (kt > kb || kk > 0) ? 1u : 0u;
                if constexpr (KIND == Kind::I8)
                  mma_i8(d_base, ad, bd, idesc2, acc);
                else
                  mma_bf16(d_base, ad, bd, idesc2, acc);
              }
              commit(&empty[s]);
              continue;
            }
          }
#pragma unroll
          for (int p = 0; p < P; ++p) {
            const uint32_t a_addr = smem_u32(st + p * S::kATile);
            const uint32_t b_addr = smem_u32(st + P * S::kATile + p * S::kBTile);
            const uint32_t d_tmem = d_base + p * BN;
#pragma unroll
            for (int kk = 0; kk < 128 / 32; ++kk) {  // 4 MMAs of 32 bytes of K each
              const uint64_t ad = smem_desc_sw128(a_addr + kk * 32);
              const uint64_t bd = smem_desc_sw128(b_addr + kk * 32);
              const uint32_t acc = (kt > kb || kk > 0) ? 1u : 0u;
              if constexpr (CG == 2) {
                if constexpr (KIND == Kind::I8)
                  mma_i8_pair(d_tmem, ad, bd, idesc, acc);
                else
                  mma_bf16_pair(d_tmem, ad, bd, idesc, acc);
              } else if constexpr (KIND == Kind::I8) {
                mma_i8(d_tmem, ad, bd, idesc, acc);
              } else {
                mma_bf16(d_tmem, ad, bd, idesc, acc);
              }
            }
          }
          commit(&empty[s]);  // stage s free (in both CTAs) once these MMAs have read it
        }
        commit(&tfull[ab]);  // the tile's accumulator is complete
        if (lt == 0) stamp(args.dbg, 5);
      }
    }
  } else if (warp < 2 + kEpiWarps) {
    // ---------------- epilogue warps 2..9
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int part = (warp - 2) / 4;  // which share of the tile's columns (kEpiWarps / 4 shares)
    const int etid = threadIdx.x - 64;  // 0 .. 32*kEpiWarps-1
    float* const_base = reinterpret_cast<float*>(smem + S::kConstOff);
    uint32_t lt = 0;
    bool ok = true;
    // Per-tile column constants (weight scale and bias of each linear of the tile, and for GeluQuant the
    // next linear's smooth vector and its reciprocal), one column per thread (BN <= epilogue threads):
    // fetched from global memory into registers one tile ahead, so their latency hides behind the current
    // tile's epilogue, and written into the constant buffer of the tile's parity.
    static_assert(BN <= 32 * kEpiWarps, "one column of constants per epilogue thread");
    float cpre[S::kConstArrays];
    auto fetch_consts = [&](int t) {
      if (t >= n_tiles_total || etid >= BN) return;
      int si, m0, n0;
      tile_coord<BN, P, CG>(args, t, si, m0, n0, rank);
      const int n = n0 + etid;
#pragma unroll
      for (int set = 0; set < P; ++set) {
        const GemmSeg& g = args.seg[P == 1 ? si : set];
        const bool in = n < g.n;
        cpre[2 * set] = (KIND == Kind::I8 && g.wscale && in) ? g.wscale[n] : 1.0f;
        cpre[2 * set + 1] = (g.bias && in) ? __bfloat162float(g.bias[n]) : -0.0f;  // x + -0 == x for every x
      }
      if constexpr (EPI == Epi::GeluQuant) {
        const bool in = args.qout && n < args.seg[si].n;
        cpre[4] = in ? args.q_smooth[n] : 1.0f;
        cpre[5] = (in && args.q_rsmooth) ? args.q_rsmooth[n] : 1.0f;
      }
    };
    auto put_consts = [&](int t, uint32_t buf) {
      if (t >= n_tiles_total || etid >= BN) return;
      float* cst = const_base + buf * S::kConstArrays * BN;
#pragma unroll
      for (int set = 0; set < P; ++set) {
        cst[(2 * set) * BN + etid] = cpre[2 * set];
        cst[(2 * set + 1) * BN + etid] = cpre[2 * set + 1];
      }
      if constexpr (EPI == Epi::GeluQuant) {
        cst[4 * BN + etid] = cpre[4];
        cst[5 * BN + etid] = cpre[5];
      }
    };
    // scales and biases are written with the weights: when those predate the previous kernel the first
    // tile's constants are requested before waiting for it
    if (args.weights_resident) fetch_consts(cl);
    pdl_wait();  // residuals / outputs may be touched by the previous kernel
    if (!args.weights_resident) fetch_consts(cl);
    put_consts(cl, 0);
    asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
    if (etid == 0) stamp(args.dbg, 6);
    // Every epilogue warp runs every iteration (also after a failed wait) so that the named barrier
    // below is reached the same number of times by all of them.
    const uint32_t tempty_leader[2] = {leader_bar(&tempty[0]), leader_bar(&tempty[1])};
    for (int t = cl; t < n_tiles_total; t += n_cl, ++lt) {
      const uint32_t ab = lt & 1, use = lt >> 1;
      int si, m0, n0;
      tile_coord<BN, P, CG>(args, t, si, m0, n0, rank);
      // this tile's constants are in buffer ab (written before the barrier that ended the previous
      // iteration); the next tile's are requested now
      const float* cst = const_base + ab * S::kConstArrays * BN;
      fetch_consts(t + n_cl);
      bool acc_waited = false, acc_ok = true;
      auto wait_acc = [&]() -> bool {
        if (acc_waited) return acc_ok;
        acc_ok = __all_sync(0xffffffffu, bounded_wait(&tfull[ab], use & 1));
        tc_fence_after();
        acc_waited = true;
        if (lt == 0 && etid == 0) stamp(args.dbg, 7);
        return acc_ok;
      };
      const uint32_t t_row = tmem_base + ab * S::kAccCols + (static_cast<uint32_t>(q * 32) << 16);
      bool run_epi = true;
      if constexpr (BN == 64) {  // split-K is compiled for the narrow tile only (the one few-tile GEMMs use)
        if (args.splits > 1) run_epi = splitk_reduce<KIND, BN, P, kEpiWarps / 4>(args, t, m0, row, part, etid, t_row, ok, split_last, wait_acc);
      }
      const bool ok_t = run_epi ? epilogue_tile<KIND, BN, P, EPI, kEpiWarps / 4>(args, si, m0, n0, t_row, row, part, ok, cst, wait_acc)
                                : (ok && acc_ok);
      if (lt == 0 && etid == 0) stamp(args.dbg, 8);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (CG == 2)
          mbar_arrive_cluster(tempty_leader[ab]);
        else
          mbar_arrive(&tempty[ab]);
      }
      ok = ok_t;
      // the other buffer was last read by the previous tile, which every warp finished before the barrier
      // that ended the previous iteration
      put_consts(t + n_cl, ab ^ 1u);
      asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory");
    }
  } else if constexpr (T::kConvert) {
    // ---------------- W8A16 weight conversion, warps 10..13, all four on every stage:
    // P x [BN rows x 64 int8] staging -> P x [BN rows x 64 bf16(q * w_s[n])] in the 128B-swizzled operand
    // layout.  The conversion uses integer / FMA arithmetic only (exact small-int -> fp32, fp32 multiply,
    // integer round-to-nearest-even), which keeps it off the slow conversion unit.
    const int et = (warp - 2 - kEpiWarps) * 32 + lane;  // 0..127
    constexpr int kPer = BN * 4 / 128;                   // (row, 16-byte chunk) items per thread and stage
    uint32_t g = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles_total && ok; t += gridDim.x) {
      int si, m0, n0;
      tile_coord<BN, P>(args, t, si, m0, n0);
      float wsr[P][kPer];  // the weight scales of this thread's rows, loaded once per tile
#pragma unroll
      for (int p = 0; p < P; ++p) {
        const GemmSeg& sp = args.seg[P == 1 ? si : p];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          const int gn = n0 + ((et + i * 128) >> 2);
          wsr[p][i] = (sp.wscale != nullptr && gn < sp.n) ? sp.wscale[gn] : 1.0f;
        }
      }
      int kb, ke;
      k_range(args, t, k_tiles, kb, ke);
      for (int kt = kb; kt < ke; ++kt, ++g) {
        const int s = g % STAGES;
        const uint32_t ph = (g / STAGES) & 1;
        ok = __all_sync(0xffffffffu, bounded_wait(&full[s], ph));
        if (!ok) break;
        uint8_t* st = smem + s * S::kStage;
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const int8_t* raw = reinterpret_cast<const int8_t*>(st + P * (S::kATile + S::kBTile) + p * S::kRawTile);
          uint8_t* bt = st + P * S::kATile + p * S::kBTile;
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int idx = et + i * 128;
            const int r = idx >> 2, c = idx & 3;
            const float ws = wsr[p][i];
            const int4 v = *reinterpret_cast<const int4*>(raw + r * 64 + c * 16);
            const int8_t* b8 = reinterpret_cast<const int8_t*>(&v);
            uint32_t packed[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t lo = bf16_rn_bits(__fmul_rn(small_int_to_f32(b8[2 * j]), ws));
              const uint32_t hi = bf16_rn_bits(__fmul_rn(small_int_to_f32(b8[2 * j + 1]), ws));
              packed[j] = __byte_perm(lo, hi, 0x7632);
            }
            // logical 16-byte chunks 2c and 2c+1 of row r, 128B swizzle: chunk ^ (r & 7)
            const int c0 = (2 * c) ^ (r & 7), c1 = (2 * c + 1) ^ (r & 7);
            *reinterpret_cast<int4*>(bt + r * 128 + c0 * 16) = make_int4(packed[0], packed[1], packed[2], packed[3]);
            *reinterpret_cast<int4*>(bt + r * 128 + c1 * 16) = make_int4(packed[4], packed[5], packed[6], packed[7]);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[s]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // a pair: neither CTA leaves while the other may still arrive on its barriers or read its shared memory
  if constexpr (CG == 2) cluster_sync();
  if (threadIdx.x == 0) stamp(args.dbg, 9);
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    if constexpr (CG == 2)
      tmem_dealloc_pair(tmem_base, S::kTmemCols);
    else
      tmem_dealloc(tmem_base, S::kTmemCols);
    if (lane == 0) stamp(args.dbg, 10);
  }
}

}  // namespace svla
