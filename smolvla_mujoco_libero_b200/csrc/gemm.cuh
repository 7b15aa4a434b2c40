// tcgen05 GEMM for sm_100a:  D[M, N] = A[M, K] * B[N, K]^T  (both operands K-major), with fused epilogues.
//
// Operand kinds
//   I8     A int8 (TMA), B int8 (TMA), tcgen05.mma kind::i8 -> int32 in TMEM.   SmoothQuant W8A8 linears.
//   BF16   A bf16 (TMA), B bf16 (TMA), kind::f16 -> fp32 in TMEM.               plain bf16 linears.
//   W8A16  A bf16 (TMA), B int8 (TMA into a staging buffer), converted by the epilogue warps to
//          bf16(q * w_s[n]) in the 128B-swizzled layout the MMA reads, then kind::f16.  W8A16 linears.
//
// CTA = 192 threads: warp 0 issues TMA, warp 1 owns TMEM and issues MMA (one elected lane), warps 2-5
// run the epilogue (TMEM lanes 32*(warp%4) .. +31) and, for W8A16, the weight conversion during the
// main loop.  Tile: 128 rows (M) x BN columns (N) x 128 bytes of K per pipeline stage.
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
  // output row remap: row = (m / rows_per_group) * group_stride + (m % rows_per_group) + row_offset
  int rows_per_group, group_stride, row_offset;
  float post_scale;                 // Bf16: multiply bf16(y) by this and round again (0 = off)
  const __nv_bfloat16* resid;       // Resid: residual rows (may alias out)
  int ldr, resid_rows;              // resid row = (resid_rows > 0 ? m % resid_rows : remapped row)
  const float2* rope_cs;            // [max_pos][32] (cos, sin)
  const int* pos;                   // [M] positions
  int max_pos;
  const float* q_smooth;            // GeluQuant: smooth vector of the next linear [N]
  float q_act;                      // GeluQuant: activation scale of the next linear
  int8_t* qout;                     // GeluQuant: int8 output [M, ldq]
  int ldq;
  float dt;                         // Euler
  float* xt;                        // Euler: fp32 state [M, ldo]
  __nv_bfloat16* xt_bf16;           // Euler: bf16 copy
  int* err;
};

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

template <Kind KIND, int BN, int P, int STAGES>
struct GemmSmem {
  static constexpr int kATile = 128 * 128;            // bytes
  static constexpr int kBTile = BN * 128;             // bytes (bf16 or int8 MMA operand)
  static constexpr int kRawTile = KindTraits<KIND>::kConvert ? BN * 64 : 0;  // int8 staging, W8A16
  static constexpr int kStage = P * (kATile + kBTile + kRawTile);
  static constexpr int kBarOff = STAGES * kStage;
  static constexpr int kBytes = kBarOff + 256 + 1024;  // barriers + alignment slack
  static constexpr int kTmemCols = (P * BN <= 32) ? 32 : (P * BN <= 64) ? 64 : (P * BN <= 128) ? 128
                                                     : (P * BN <= 256) ? 256 : 512;
};

__device__ __forceinline__ float silu_f(float x) { return __fdiv_rn(x, 1.0f + expf(-x)); }

__device__ __forceinline__ float gelu_tanh_f(float x) {
  // 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 x^3)))
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  float inner = k0 * (x + k1 * x * x * x);
  return 0.5f * x * (1.0f + tanhf(inner));
}

template <Kind KIND, int BN, int P, int STAGES, Epi EPI>
__global__ void __launch_bounds__(192, 1) gemm_sm100_kernel(const __grid_constant__ GemmArgs args) {
  using T = KindTraits<KIND>;
  using S = GemmSmem<KIND, BN, P, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;          // W8A16: converted B ready
  uint64_t* accum = conv + STAGES;          // all MMAs done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tile = blockIdx.x;
  const int n_tile = blockIdx.y;

  // segment lookup
  int si = 0;
  if constexpr (P == 1) {
#pragma unroll
    for (int s = 1; s < 3; ++s)
      if (s < args.nseg && n_tile >= args.seg[s].tile_begin) si = s;
  }
  const GemmSeg& sg = args.seg[si];
  const int n0 = (n_tile - sg.tile_begin) * BN;  // first column within the segment
  const int m0 = m_tile * 128;
  const int k_tiles = (args.K + T::kBK - 1) / T::kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&conv[s], 4);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

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
      for (int p = 0; p < P; ++p) {
        prefetch_tmap(&args.ta[P == 1 ? si : p]);
        prefetch_tmap(&args.tb[P == 1 ? si : p]);
      }
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        if (!bounded_wait(&empty[s], ph ^ 1)) break;
        uint8_t* st = smem + s * S::kStage;
        constexpr uint32_t kBBytes = T::kConvert ? S::kRawTile : S::kBTile;
        mbar_arrive_expect_tx(&full[s], P * (S::kATile + kBBytes));
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const int mi = (P == 1) ? si : p;
          uint8_t* a_dst = st + p * S::kATile;
          uint8_t* b_dst = T::kConvert ? st + P * (S::kATile + S::kBTile) + p * S::kRawTile
                                       : st + P * S::kATile + p * S::kBTile;
          tma_load_2d(a_dst, &args.ta[mi], &full[s], kt * T::kBK, m0);
          tma_load_2d(b_dst, &args.tb[mi], &full[s], kt * T::kBK, n0);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t idesc = T::idesc(BN);
      bool ok = true;
      for (int kt = 0; kt < k_tiles && ok; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        ok = bounded_wait(&full[s], ph);
        if (ok && T::kConvert) ok = bounded_wait(&conv[s], ph);
        if (!ok) break;
        tc_fence_after();
        uint8_t* st = smem + s * S::kStage;
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const uint32_t a_addr = smem_u32(st + p * S::kATile);
          const uint32_t b_addr = smem_u32(st + P * S::kATile + p * S::kBTile);
          const uint32_t d_tmem = tmem_base + p * BN;
#pragma unroll
          for (int kk = 0; kk < 128 / 32; ++kk) {  // 4 MMAs of 32 bytes of K each
            {
              const uint64_t ad = smem_desc_sw128(a_addr + kk * 32);
              const uint64_t bd = smem_desc_sw128(b_addr + kk * 32);
              const uint32_t acc = (kt > 0 || kk > 0) ? 1u : 0u;
              if constexpr (KIND == Kind::I8)
                mma_i8(d_tmem, ad, bd, idesc, acc);
              else
                mma_bf16(d_tmem, ad, bd, idesc, acc);
            }
          }
        }
        mma_commit(&empty[s]);  // stage s free once these MMAs have read it
      }
      mma_commit(accum);  // arrives when every MMA issued above has completed
    }
  } else {
    // ---------------- epilogue warps (2..5); W8A16 weight conversion during the main loop
    const int q = warp & 3;      // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int et = (warp - 2) * 32 + lane;  // 0..127
    if constexpr (T::kConvert) {
      // each stage: P x [BN rows x 64 int8] staging -> P x [BN rows x 64 bf16] swizzled operand tiles
      for (int kt = 0; kt < k_tiles; ++kt) {
        const int s = kt % STAGES;
        const uint32_t ph = (kt / STAGES) & 1;
        const bool okc = bounded_wait(&full[s], ph);
        if (!__all_sync(0xffffffffu, okc)) break;
        uint8_t* st = smem + s * S::kStage;
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const GemmSeg& sp = args.seg[P == 1 ? si : p];
          const int8_t* raw = reinterpret_cast<const int8_t*>(st + P * (S::kATile + S::kBTile) + p * S::kRawTile);
          uint8_t* bt = st + P * S::kATile + p * S::kBTile;
          // BN rows x 4 chunks of 16 int8 -> 8 chunks of 16 bytes of bf16
          for (int idx = et; idx < BN * 4; idx += 128) {
            const int r = idx >> 2, c = idx & 3;
            const int gn = n0 + r;
            const float ws = (sp.wscale != nullptr && gn < sp.n) ? sp.wscale[gn] : 1.0f;
            const int4 v = *reinterpret_cast<const int4*>(raw + r * 64 + c * 16);
            const int8_t* b8 = reinterpret_cast<const int8_t*>(&v);
            uint32_t packed[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              __nv_bfloat162 h;
              h.x = __float2bfloat16_rn(__fmul_rn(static_cast<float>(b8[2 * j]), ws));
              h.y = __float2bfloat16_rn(__fmul_rn(static_cast<float>(b8[2 * j + 1]), ws));
              packed[j] = *reinterpret_cast<uint32_t*>(&h);
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

    // wait for the accumulator
    const bool ok = __all_sync(0xffffffffu, bounded_wait(accum, 0));
    tc_fence_after();
    const int m = m0 + row;
    const bool row_ok = ok && (m < args.M);
    int orow = m;
    if (args.rows_per_group > 0) orow = (m / args.rows_per_group) * args.group_stride + (m % args.rows_per_group);
    orow += args.row_offset;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16);

    auto dequant = [&](const GemmSeg& g, uint32_t raw, int n) -> float {
      float v;
      if constexpr (KIND == Kind::I8) {
        v = __fmul_rn(static_cast<float>(static_cast<int>(raw)), g.act_scale);
        if (g.wscale) v = __fmul_rn(v, g.wscale[n]);
      } else {
        v = __uint_as_float(raw);
      }
      if (g.bias) v = __fadd_rn(v, __bfloat162float(g.bias[n]));
      if (g.bias_f32) v = __fadd_rn(v, g.bias_f32[n]);
      return v;
    };

    if constexpr (EPI == Epi::Rope) {
      // 64 columns (one head) at a time
      for (int c = 0; c < BN; c += 64) {
        uint32_t r[64];
        if (ok) {
          tmem_ld16(t_row + c, *reinterpret_cast<uint32_t(*)[16]>(&r[0]));
          tmem_ld16(t_row + c + 16, *reinterpret_cast<uint32_t(*)[16]>(&r[16]));
          tmem_ld16(t_row + c + 32, *reinterpret_cast<uint32_t(*)[16]>(&r[32]));
          tmem_ld16(t_row + c + 48, *reinterpret_cast<uint32_t(*)[16]>(&r[48]));
          tmem_ld_wait();
        }
        const int nb = n0 + c;
        if (!row_ok || nb >= sg.n) continue;
        float v[64];
#pragma unroll
        for (int j = 0; j < 64; ++j) v[j] = bf16_round(dequant(sg, r[j], nb + j));
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb;
        if (sg.rope) {
          int p = args.pos[m];
          p = p < 0 ? 0 : (p >= args.max_pos ? args.max_pos - 1 : p);
          const float2* cs = args.rope_cs + static_cast<size_t>(p) * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float2 t = cs[j];
            const float x1 = v[j], x2 = v[j + 32];
            const float o1 = __fsub_rn(__fmul_rn(x1, t.x), __fmul_rn(x2, t.y));
            const float o2 = __fadd_rn(__fmul_rn(x2, t.x), __fmul_rn(x1, t.y));
            v[j] = o1;
            v[j + 32] = o2;
          }
        }
#pragma unroll
        for (int j = 0; j < 64; j += 8) {
          uint32_t pk[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[j + 2 * u], v[j + 2 * u + 1]);
            pk[u] = *reinterpret_cast<uint32_t*>(&h);
          }
          *reinterpret_cast<int4*>(o + j) = make_int4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
    } else {
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16], r2[16];
        if (ok) {
          tmem_ld16(t_row + c, r);
          if constexpr (P == 2) tmem_ld16(t_row + BN + c, r2);
          tmem_ld_wait();
        }
        const int nb = n0 + c;
        if (!row_ok || nb >= sg.n) continue;
        if constexpr (EPI == Epi::I32) {
          int* o = reinterpret_cast<int*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb;
#pragma unroll
          for (int j = 0; j < 16; j += 4) *reinterpret_cast<int4*>(o + j) = make_int4(r[j], r[j + 1], r[j + 2], r[j + 3]);
        } else if constexpr (EPI == Epi::F32) {
          float* o = reinterpret_cast<float*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb;
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(o + j) = make_float4(dequant(sg, r[j], nb + j), dequant(sg, r[j + 1], nb + j + 1),
                                                            dequant(sg, r[j + 2], nb + j + 2), dequant(sg, r[j + 3], nb + j + 3));
        } else if constexpr (EPI == Epi::Euler) {
          float* xo = args.xt + static_cast<size_t>(orow) * sg.ldo + nb;
          __nv_bfloat16* xb = args.xt_bf16 + static_cast<size_t>(orow) * sg.ldo + nb;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float vt = dequant(sg, r[j], nb + j);
            const float x = __fadd_rn(xo[j], __fmul_rn(args.dt, vt));
            xo[j] = x;
            xb[j] = __float2bfloat16_rn(x);
          }
        } else {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = bf16_round(dequant(sg, r[j], nb + j));
          if constexpr (EPI == Epi::SiluMul) {
            const GemmSeg& su = args.seg[1];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float u = bf16_round(dequant(su, r2[j], nb + j));
              v[j] = __fmul_rn(bf16_round(silu_f(v[j])), u);
            }
          } else if constexpr (EPI == Epi::SiluBf16) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = silu_f(v[j]);
          } else if constexpr (EPI == Epi::Resid) {
            const int rr = args.resid_rows > 0 ? (m % args.resid_rows) : orow;
            const __nv_bfloat16* rs = args.resid + static_cast<size_t>(rr) * args.ldr + nb;
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = __fadd_rn(v[j], __bfloat162float(rs[j]));
          } else if constexpr (EPI == Epi::GeluQuant) {
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = bf16_round(gelu_tanh_f(v[j]));
            if (args.qout != nullptr) {
              int8_t qv[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) qv[j] = smooth_quant(v[j], args.q_smooth[nb + j], args.q_act);
              *reinterpret_cast<int4*>(args.qout + static_cast<size_t>(orow) * args.ldq + nb) =
                  *reinterpret_cast<int4*>(qv);
            }
            if (sg.out == nullptr) continue;
          } else if constexpr (EPI == Epi::Bf16) {
            if (args.post_scale != 0.0f) {
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(v[j], args.post_scale);
            }
          }
          __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(sg.out) + static_cast<size_t>(orow) * sg.ldo + nb;
          uint32_t pk[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * u], v[2 * u + 1]);
            pk[u] = *reinterpret_cast<uint32_t*>(&h);
          }
          *reinterpret_cast<int4*>(o) = make_int4(pk[0], pk[1], pk[2], pk[3]);
          *reinterpret_cast<int4*>(o + 8) = make_int4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

}  // namespace svla
