// Persistent warp-specialized tcgen05 GEMM for sm_100a, batched over G groups:
//
//     C[g] (M x N) = A[g] (M x K) . B[g] (N x K)^T        (fp32 accumulate in TMEM)
//
// Operands are bf16, staged by TMA (128-byte swizzle) from THIS GPU's memory only.
// Each operand may be K-major (reduction dim contiguous) or MN-major (row dim
// contiguous), so a Linear's forward (X W^T), input gradient (dY W) and weight
// gradient (dY^T X) all map onto this one kernel without transposed copies.
//
// CTA = 6 warps: warp 0 issues TMA loads into an S-stage ring, warp 1 owns TMEM
// and issues tcgen05.mma from one thread (128 x BN x 16 per instruction), warps 2-5
// drain a double-buffered TMEM accumulator (2 x BN fp32 columns) through a fused
// epilogue while the next tile's MMAs run. Tiles are distributed round-robin over a
// persistent grid of one CTA per SM.
//
// Epilogues (template EPI):
//   EPI_BF16     C = bf16(acc)
//   EPI_F32      C = acc + beta * C                         (fp32)
//   EPI_RESID    C = R + acc                                (fp32 residual stream)
//   EPI_SWIGLU   B tile = [gate rows | up rows] of one 64-feature block;
//                H = bf16(silu(bf16 g) * bf16 u), GU aux = bf16 g, u
//   EPI_SWIGLU_BWD  acc = dH; reads g,u; writes dG, dU (bf16) into C = [dG | dU]
//   EPI_LOGITS   C = bf16(acc) and per-row (max, sum exp) of the rounded tile values
//
// bf16 outputs of 128-wide tiles (EPI_BF16, EPI_LOGITS) are written through shared
// memory: each epilogue warp stages its 32 x 64 sub-tile in the 128-byte-swizzle layout
// and one lane issues a TMA tensor store (no multicast; the destination is this GPU's
// memory), so a warp's store is one bulk transfer instead of 32 row-strided ones.
#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {

enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_SWIGLU_BWD = 4, EPI_LOGITS = 5 };

struct GemmParams {
  int M, N, K, G;
  int tiles_m, tiles_n, num_tiles, num_kb;
  void* C;
  long long ldc, sc;
  const float* R;
  long long ldr, sr;
  void* aux;  // swiglu: pre-activation [M, 2F] bf16 ([g | u]); bwd: same layout as input
  long long ldx, sx;
  float* part;  // logits: [G][M][2 * tiles_n] float2 (one per tile column half)
  // fp32 outputs (TMA-store epilogue): sum of squares of every 32 x 32 output box, at
  // sqp[g * sq_ld + (row / 32) * ceil(N / 32) + col / 32] (each box written once)
  float* sqp;
  long long sq_ld;
  float beta;
  int f_half;  // swiglu: F (rows of the gate block; up block starts at row F)
  int tma_store;  // bf16 / logits with BN 128: stage each warp's 32 x 64 sub-tile in smem, TMA-store it
  int* err;
  // Softmax-gradient operand (gemm_ce_grad): A holds bf16 logits and is turned into the CE
  // dlogits in shared memory before the MMAs read it. xf = 1: A = logits [tokens, vocab]
  // (K-major, K = vocab; the input gradient); xf = 2: A = logits^T (MN-major, M = vocab,
  // K = tokens; the weight gradient). Per token of path g: ob = ce_ob(lse, sc) and the
  // label at xf_ob / xf_lab [g * xf_ms + token] (label < 0: row ignored), sc = xf_sc[g].
  // GEMM group gg is path gg / xf_split, token offset (gg % xf_split) * K (split-K).
  int xf;
  const float* xf_ob;
  const int* xf_lab;
  const float* xf_sc;
  long long xf_ms;
  int xf_split;
};

constexpr int BM = 128;
constexpr int BK = 64;

// TMEM columns for two accumulator buffers of width BN (allocations are powers of two).
constexpr int tmem_cols(int bn) {
  int c = 32;
  while (c < 2 * bn) c *= 2;
  return c;
}
constexpr int kThreads = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 epilogue
constexpr int kThreadsXF = 576;  // + warps 10-17: softmax-gradient transform of the A operand

// Staging bytes per epilogue warp: one 4 KB box for bf16 / logits outputs, two for the
// other epilogues of the single-CTA kernel (two fp32 boxes in flight, or the three bf16
// boxes of a SwiGLU slab).
constexpr int stg_warp_bytes(int epi, bool pair) { return (epi == EPI_BF16 || epi == EPI_LOGITS || pair) ? 4096 : 8192; }

// Pipeline depth that fits next to the staging buffers and barriers.
constexpr int fit_stages(int stage_bytes, int stg_total, int want) {
  int s = want;
  while (s > 2 && s * stage_bytes + stg_total + 512 + 1024 > 232448) --s;
  return s;
}

template <int BN, int STAGES, int STGW = 4096>
struct SmemLayout {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;  // epilogue staging: 8 warps x STGW bytes
  static constexpr int STG_BYTES = 8 * STGW;
  static constexpr int BAR_OFF = STG_OFF + STG_BYTES;
  static constexpr int TOTAL = BAR_OFF + 512 + 1024;  // + barriers + alignment slack
  static_assert(TOTAL <= 232448, "shared memory budget");
};

// Write 32 bf16 values (columns [c0, c0 + 32) of a 64-column staging row) into a
// [32 rows][64 bf16] staging buffer in the 128-byte-swizzle layout of the output map.
ODP_DEVICE void stage_bf16x32(uint8_t* stg, int row, int c0, const float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int chunk = (c0 >> 3) + j;
    uint4 w = make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                         pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
    *reinterpret_cast<uint4*>(stg + row * 128 + ((chunk ^ (row & 7)) << 4)) = w;
  }
}

// silu and the logistic function with the fast reciprocal (__fdividef: 2 ulp, far below
// the bf16 rounding that follows every use here; 0 when 1 + e^-x overflows).
ODP_DEVICE float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
ODP_DEVICE float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

// Load 32 accumulator columns [c, c+32) of this thread's TMEM lane into fp32.
ODP_DEVICE void load32(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld16_nw(taddr, r);
  tmem_ld16_nw(taddr + 16, r + 16);
  tmem_wait_tie32(r);
}

ODP_DEVICE void store_bf16x32(__nv_bfloat16* dst, const float* v) {
  uint32_t w[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2) w[i / 2] = pack_bf16(v[i], v[i + 1]);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d4[i] = make_uint4(w[4 * i], w[4 * i + 1], w[4 * i + 2], w[4 * i + 3]);
}

ODP_DEVICE void load_bf16x32(const __nv_bfloat16* src, float* v) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 q = s4[i];
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&q);
#pragma unroll
    for (int j = 0; j < 8; ++j) v[8 * i + j] = __bfloat162float(h[j]);
  }
}

// Epilogue of one tile for one thread: TMEM lane row q*32+lane, column half `ch`
// (two warps share a lane quarter; each drains BN/2 columns).
template <int BN, int EPI, int STGW = 4096>
ODP_DEVICE void epilogue_tile(const GemmParams& p, uint32_t tmem_acc, int q, int ch, int lane, int g, int tm,
                              int tn, uint8_t* stg, const CUtensorMap* tmC) {
  const int row = q * 32 + lane;
  const long long grow = (long long)tm * BM + row;
  const bool row_ok = grow < p.M;
  const uint32_t tbase = tmem_acc + ((uint32_t)(q * 32) << 16);
  constexpr int HALF = BN / 2;

  if constexpr (EPI == EPI_SWIGLU) {
    // columns [0, HALF) = gate block, [HALF, BN) = up block of the same HALF features;
    // this thread takes HALF/2 of them.
    constexpr int QW = HALF / 2;
    static_assert(QW == 32, "swiglu epilogue expects BN == 128");
    const int c0 = ch * QW;
    const int f0 = tn * HALF + c0;
    uint32_t a[32], b[32];
    tmem_ld16_nw(tbase + c0, a);
    tmem_ld16_nw(tbase + c0 + 16, a + 16);
    tmem_ld16_nw(tbase + HALF + c0, b);
    tmem_ld16_nw(tbase + HALF + c0 + 16, b + 16);
    tmem_wait_tie32(a);
    reg_tie32(b);
    if (!row_ok || f0 >= p.f_half) return;
    float h[32], gg[32], uu[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      gg[i] = bf16_round(__uint_as_float(a[i]));
      uu[i] = bf16_round(__uint_as_float(b[i]));
      h[i] = bf16_round(silu_f(gg[i])) * uu[i];
    }
    __nv_bfloat16* H = reinterpret_cast<__nv_bfloat16*>(p.C) + g * p.sc + grow * p.ldc + f0;
    __nv_bfloat16* GU = reinterpret_cast<__nv_bfloat16*>(p.aux) + g * p.sx + grow * p.ldx + f0;
    store_bf16x32(H, h);
    store_bf16x32(GU, gg);
    store_bf16x32(GU + p.f_half, uu);
  } else {
    if constexpr (EPI == EPI_BF16 && (BN == 128 || BN == 256) && STGW >= (BN / 2) * 64) {
      if (p.tma_store) {
        // every box of this warp's 32 x HALF slab staged at once: one proxy fence, then
        // one TMA store per box (the buffer is free again once the previous tile's stores
        // have been read out, long before)
        if (lane == 0) bulk_wait_read0();
        __syncwarp();
#pragma unroll 1
        for (int b = 0; b < HALF; b += 64)
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            uint32_t r[32];
            load32(tbase + ch * HALF + b + c, r);
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            stage_bf16x32(stg + (b / 64) * 4096, lane, c, v);
          }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int b = 0; b < HALF; b += 64)
            tma_store_3d(tmC, stg + (b / 64) * 4096, tn * BN + ch * HALF + b, tm * BM + q * 32, g);
          bulk_commit();
        }
        __syncwarp();
        return;
      }
    } else if constexpr (EPI == EPI_BF16 && (BN == 128 || BN == 256)) {
      if (p.tma_store) {
#pragma unroll 1
        for (int b = 0; b < HALF; b += 64) {  // one 32 x 64 box at a time through the 4 KB buffer
          // the previous box stored from this buffer must have been read out
          if (lane == 0) bulk_wait_read0();
          __syncwarp();
#pragma unroll 1
          for (int c = 0; c < 64; c += 32) {
            uint32_t r[32];
            load32(tbase + ch * HALF + b + c, r);
            float v[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
            stage_bf16x32(stg, lane, c, v);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(tmC, stg, tn * BN + ch * HALF + b, tm * BM + q * 32, g);
            bulk_commit();
          }
          __syncwarp();
        }
        return;
      }
    }
#pragma unroll 1
    for (int c = ch * HALF; c < (ch + 1) * HALF; c += 32) {
      uint32_t r[32];
      load32(tbase + c, r);
      const int gcol = tn * BN + c;
      if (!row_ok || gcol >= p.N) continue;
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      const bool full = gcol + 32 <= p.N;
      if constexpr (EPI == EPI_BF16) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + g * p.sc + grow * p.ldc + gcol;
        if (full) store_bf16x32(dst, v);
        else for (int i = 0; gcol + i < p.N; ++i) dst[i] = __float2bfloat16(v[i]);
      } else if constexpr (EPI == EPI_SWIGLU_BWD) {
        // acc = dH (gradient of silu(g) * u); aux = saved [g | u]; C = [dG | dU]
        const __nv_bfloat16* gsrc = reinterpret_cast<const __nv_bfloat16*>(p.aux) + g * p.sx + grow * p.ldx + gcol;
        __nv_bfloat16* dg = reinterpret_cast<__nv_bfloat16*>(p.C) + g * p.sc + grow * p.ldc + gcol;
        float gv[32], uv[32], og[32], ou[32];
        if (full) {
          load_bf16x32(gsrc, gv);
          load_bf16x32(gsrc + p.f_half, uv);
        } else {
          for (int i = 0; i < 32; ++i) {
            gv[i] = gcol + i < p.N ? __bfloat162float(gsrc[i]) : 0.f;
            uv[i] = gcol + i < p.N ? __bfloat162float(gsrc[p.f_half + i]) : 0.f;
          }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float dh = bf16_round(v[i]);
          const float sg = sigmoid_f(gv[i]);
          ou[i] = dh * bf16_round(gv[i] * sg);
          og[i] = bf16_round(dh * uv[i]) * sg * (1.0f + gv[i] * (1.0f - sg));
        }
        if (full) {
          store_bf16x32(dg, og);
          store_bf16x32(dg + p.f_half, ou);
        } else {
          for (int i = 0; gcol + i < p.N; ++i) {
            dg[i] = __float2bfloat16(og[i]);
            dg[p.f_half + i] = __float2bfloat16(ou[i]);
          }
        }
      } else if constexpr (EPI == EPI_F32 || EPI == EPI_RESID) {
        float* dst = reinterpret_cast<float*>(p.C) + g * p.sc + grow * p.ldc + gcol;
        if (full) {
          float4* d4 = reinterpret_cast<float4*>(dst);
          if constexpr (EPI == EPI_RESID) {
            const float4* r4 = reinterpret_cast<const float4*>(p.R + g * p.sr + grow * p.ldr + gcol);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 x = r4[i];
              d4[i] = make_float4(x.x + v[4 * i], x.y + v[4 * i + 1], x.z + v[4 * i + 2], x.w + v[4 * i + 3]);
            }
          } else {
            if (p.beta != 0.f) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                float4 x = d4[i];
                d4[i] = make_float4(v[4 * i] + p.beta * x.x, v[4 * i + 1] + p.beta * x.y,
                                    v[4 * i + 2] + p.beta * x.z, v[4 * i + 3] + p.beta * x.w);
              }
            } else {
#pragma unroll
              for (int i = 0; i < 8; ++i) d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
            }
          }
        } else {
          for (int i = 0; gcol + i < p.N; ++i) {
            float x = v[i];
            if constexpr (EPI == EPI_RESID) x += p.R[g * p.sr + grow * p.ldr + gcol + i];
            else if (p.beta != 0.f) x += p.beta * dst[i];
            dst[i] = x;
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------- TMA-store epilogues
// Each epilogue warp owns 32 TMEM lanes (rows) of the tile and a private staging buffer
// of kStgWarp bytes. A thread holds one row, so it writes its row into the buffer in the
// swizzled layout of the output tensor map, and one elected lane moves the whole 32-row
// box with a bulk tensor store (full-line writes instead of 32 scattered rows per
// instruction). Inputs of the epilogue (residual, saved gate/up pre-activations, C when
// beta != 0) come in the same way, by a TMA load on the warp's own mbarrier.
//   fp32 box: 32 rows x 32 floats (128-byte rows, 128-byte swizzle: chunk ^ row % 8)
//   bf16 box: 32 rows x 32 bf16  (64-byte rows, 64-byte swizzle: chunk ^ (row / 2) % 4)
ODP_DEVICE uint32_t f32_slot(int row, int j) { return row * 128 + ((j ^ (row & 7)) << 4); }
ODP_DEVICE uint32_t b16_slot(int row, int j) { return row * 64 + ((j ^ ((row >> 1) & 3)) << 4); }

ODP_DEVICE void stage_f32x32(uint8_t* buf, int row, const float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<float4*>(buf + f32_slot(row, j)) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
}
ODP_DEVICE void unstage_f32x32(const uint8_t* buf, int row, float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float4 x = *reinterpret_cast<const float4*>(buf + f32_slot(row, j));
    v[4 * j] = x.x;
    v[4 * j + 1] = x.y;
    v[4 * j + 2] = x.z;
    v[4 * j + 3] = x.w;
  }
}
ODP_DEVICE void stage_b16x32(uint8_t* buf, int row, const float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j)
    *reinterpret_cast<uint4*>(buf + b16_slot(row, j)) =
        make_uint4(pack_bf16(v[8 * j], v[8 * j + 1]), pack_bf16(v[8 * j + 2], v[8 * j + 3]),
                   pack_bf16(v[8 * j + 4], v[8 * j + 5]), pack_bf16(v[8 * j + 6], v[8 * j + 7]));
}
ODP_DEVICE void unstage_b16x32(const uint8_t* buf, int row, float* v) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint4 q = *reinterpret_cast<const uint4*>(buf + b16_slot(row, j));
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[8 * j + 2 * e] = __uint_as_float(w[e] << 16);
      v[8 * j + 2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
    }
  }
}

template <int N>
ODP_DEVICE void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

struct EpiCtx {
  uint8_t* stg;              // this warp's staging buffer (stg_bytes)
  int stg_bytes;
  uint64_t* wbar;            // this warp's mbarrier for epilogue inputs
  uint32_t* wphase;          // its phase parity
  const CUtensorMap* tmC;    // output map
  const CUtensorMap* tmX;    // input map (residual / saved gate-up / C)
};

// Warp-collective: bring `nbox` boxes of `box_bytes` at (x_i, y) into buf + i * box_bytes.
ODP_DEVICE bool epi_load(const GemmParams& p, EpiCtx& e, uint8_t* buf, int nbox, int box_bytes, const int* xs, int y,
                         int g, int lane) {
  if (lane == 0) {
    mbar_expect_tx(e.wbar, (uint32_t)(nbox * box_bytes));
    for (int i = 0; i < nbox; ++i) tma_load_3d(e.tmX, e.wbar, buf + i * box_bytes, xs[i], y, g);
  }
  __syncwarp();
  bool ok = mbar_wait(e.wbar, *e.wphase, p.err, ERR_TIMEOUT_FULL);
  if (!ok) ok = mbar_wait(e.wbar, *e.wphase, p.err, ERR_TIMEOUT_FULL);  // drain: a late copy must land first
  *e.wphase ^= 1u;
  return __all_sync(0xffffffffu, ok);
}

// Warp-collective: make the staged rows visible to the async proxy and store the boxes.
ODP_DEVICE void epi_store(EpiCtx& e, const CUtensorMap* m, const uint8_t* buf, int nbox, int box_bytes, const int* xs,
                          int y, int g, int lane) {
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    for (int i = 0; i < nbox; ++i) tma_store_3d(m, buf + i * box_bytes, xs[i], y, g);
    bulk_commit();
  }
  __syncwarp();
}

// Returns false when an input box never arrived (error recorded): the caller stops.
template <int BN, int EPI>
ODP_DEVICE bool epilogue_tma(const GemmParams& p, uint32_t tmem_acc, int q, int ch, int lane, int g, int tm, int tn,
                             EpiCtx& e) {
  const uint32_t tbase = tmem_acc + ((uint32_t)(q * 32) << 16);
  const int y = tm * BM + q * 32;  // first row of this warp's box (rows >= M are clipped)
  constexpr int HALF = BN / 2;
  if constexpr (EPI == EPI_SWIGLU) {
    // gate columns [0, HALF), up columns [HALF, BN) of HALF features; this warp: 32 of them
    const int c0 = ch * 32;
    const int f0 = tn * HALF + c0;
    uint32_t a[32], b[32];
    tmem_ld16_nw(tbase + c0, a);
    tmem_ld16_nw(tbase + c0 + 16, a + 16);
    tmem_ld16_nw(tbase + HALF + c0, b);
    tmem_ld16_nw(tbase + HALF + c0 + 16, b + 16);
    tmem_wait_tie32(a);
    reg_tie32(b);
    if (f0 >= p.f_half) return true;
    float h[32], gg[32], uu[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      gg[i] = bf16_round(__uint_as_float(a[i]));
      uu[i] = bf16_round(__uint_as_float(b[i]));
      h[i] = bf16_round(silu_f(gg[i])) * uu[i];
    }
    if (lane == 0) bulk_wait_read<0>();  // the previous tile's boxes have left the buffer
    __syncwarp();
    stage_b16x32(e.stg, lane, h);
    stage_b16x32(e.stg + 2048, lane, gg);
    stage_b16x32(e.stg + 4096, lane, uu);
    const int xh[1] = {f0}, xgu[2] = {f0, p.f_half + f0};
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(e.tmC, e.stg, xh[0], y, g);
      tma_store_3d(e.tmX, e.stg + 2048, xgu[0], y, g);
      tma_store_3d(e.tmX, e.stg + 4096, xgu[1], y, g);
      bulk_commit();
    }
    __syncwarp();
  } else if constexpr (EPI == EPI_SWIGLU_BWD) {
    // acc = dH for features [tn * BN + ch * HALF, + HALF); aux = saved [g | u]; C = [dG | dU]
#pragma unroll 1
    for (int c = ch * HALF; c < (ch + 1) * HALF; c += 32) {
      uint32_t r[32];
      load32(tbase + c, r);
      const int f = tn * BN + c;
      if (f >= p.N) continue;
      if (lane == 0) bulk_wait_read<0>();
      __syncwarp();
      const int xs[2] = {f, p.f_half + f};
      if (!epi_load(p, e, e.stg, 2, 2048, xs, y, g, lane)) return false;
      float gv[32], uv[32], og[32], ou[32];
      unstage_b16x32(e.stg, lane, gv);
      unstage_b16x32(e.stg + 2048, lane, uv);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float dh = bf16_round(__uint_as_float(r[i]));
        const float sg = sigmoid_f(gv[i]);
        ou[i] = dh * bf16_round(gv[i] * sg);
        og[i] = bf16_round(dh * uv[i]) * sg * (1.0f + gv[i] * (1.0f - sg));
      }
      stage_b16x32(e.stg, lane, og);
      stage_b16x32(e.stg + 2048, lane, ou);
      epi_store(e, e.tmC, e.stg, 2, 2048, xs, y, g, lane);
    }
  } else {
    // fp32 C = acc (+ R for the residual epilogue, + beta * C when beta != 0)
    const bool need_in = EPI == EPI_RESID || p.beta != 0.f;
    const int nslot = e.stg_bytes / 4096;
    int used = 0;
#pragma unroll 1
    for (int c = ch * HALF; c < (ch + 1) * HALF; c += 32) {
      uint32_t r[32];
      load32(tbase + c, r);
      float v[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
      const int slot = used % nslot;
      uint8_t* buf = e.stg + slot * 4096;
      // the slot's previous box has been read out (at most nslot - 1 newer groups pending)
      if (lane == 0) {
        if (nslot == 1) bulk_wait_read<0>();
        else bulk_wait_read<1>();
      }
      __syncwarp();
      const int xs[1] = {tn * BN + c};
      if (need_in) {
        if (!epi_load(p, e, buf, 1, 4096, xs, y, g, lane)) return false;
        float x[32];
        unstage_f32x32(buf, lane, x);
        if constexpr (EPI == EPI_RESID) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = x[i] + v[i];
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = v[i] + p.beta * x[i];
        }
      }
      if (p.sqp) {
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) q = fmaf(v[i], v[i], q);
        q = warp_sum(q);
        if (lane == 0 && y < p.M && xs[0] < p.N)
          p.sqp[(long long)g * p.sq_ld + (long long)(y / 32) * ((p.N + 31) / 32) + xs[0] / 32] = q;
      }
      stage_f32x32(buf, lane, v);
      epi_store(e, e.tmC, buf, 1, 4096, xs, y, g, lane);
      ++used;
    }
  }
  return true;
}

// Logits epilogue: bf16 store + per-row (max, sum exp) over this thread's half of the
// tile (partials indexed [row][2 * tn + ch]).
template <int BN>
ODP_DEVICE void epilogue_logits(const GemmParams& p, uint32_t tmem_acc, int q, int ch, int lane, int g, int tm,
                                int tn, uint8_t* stg, const CUtensorMap* tmC) {
  const int row = q * 32 + lane;
  const long long grow = (long long)tm * BM + row;
  const bool row_ok = grow < p.M;
  const uint32_t tbase = tmem_acc + ((uint32_t)(q * 32) << 16);
  constexpr int HALF = BN / 2;
  const bool staged = p.tma_store != 0;
  if (staged) {
    if (lane == 0) bulk_wait_read0();
    __syncwarp();
  }
  float mx = -INFINITY, se = 0.f;
#pragma unroll 1
  for (int c = ch * HALF; c < (ch + 1) * HALF; c += 32) {
    uint32_t rr[32];
    load32(tbase + c, rr);
    const int gcol = tn * BN + c;
    float r[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) r[i] = bf16_round(__uint_as_float(rr[i]));
    if (staged) stage_bf16x32(stg, lane, c - ch * HALF, r);  // out-of-range rows/cols are clipped by the map
    if (!row_ok || gcol >= p.N) continue;
    const int n = min(32, p.N - gcol);
    if (!staged) {
      __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.C) + g * p.sc + grow * p.ldc + gcol;
      if (n == 32) store_bf16x32(dst, r);
      else for (int i = 0; i < n; ++i) dst[i] = __float2bfloat16(r[i]);
    }
    float cm = -INFINITY;
#pragma unroll
    for (int i = 0; i < 32; ++i) cm = i < n ? fmaxf(cm, r[i]) : cm;
    if (cm > mx) {
      se *= __expf(mx - cm);
      mx = cm;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) se += i < n ? __expf(r[i] - mx) : 0.f;
  }
  if (staged) {
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_3d(tmC, stg, tn * BN + ch * HALF, tm * BM + q * 32, g);
      bulk_commit();
    }
    __syncwarp();
  }
  if (row_ok) {
    float2* pp = reinterpret_cast<float2*>(p.part) + ((long long)g * p.M + grow) * (2 * p.tiles_n) + 2 * tn + ch;
    *pp = make_float2(mx, se);
  }
}

template <bool A_MN, bool B_MN, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX, GemmParams p) {
  constexpr int STGW = stg_warp_bytes(EPI, false);
  using L = SmemLayout<BN, STAGES, STGW>;
  constexpr bool SPLIT_B = (EPI == EPI_SWIGLU);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* drain = accempty + 2;
  uint64_t* wbar = drain + 1;  // one per epilogue warp: inputs of the TMA-store epilogue
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(wbar + 8);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 256);
    }
    mbar_init(drain, 1);
    for (int w = 0; w < 8; ++w) mbar_init(&wbar[w], 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_holder, tmem_cols(BN));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();     // global memory only from here on
  pdl_trigger();  // after this CTA's TMEM allocation

  const int tiles_per_g = p.tiles_m * p.tiles_n;
  constexpr uint32_t kIdesc = umma_idesc_bf16(BM, BN, A_MN, B_MN);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      const int g = t / tiles_per_g, r = t % tiles_per_g;
      const int tm = r / p.tiles_n, tn = r % p.tiles_n;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, ERR_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          mbar_expect_tx(&full[stage], L::STAGE_BYTES);
          const int k0 = kb * BK;
          if constexpr (!A_MN) {
            tma_load_3d(&tmA, &full[stage], sA, k0, tm * BM, g);
          } else {
            tma_load_3d(&tmA, &full[stage], sA, tm * BM, k0, g);
            tma_load_3d(&tmA, &full[stage], sA + 8192, tm * BM + 64, k0, g);
          }
          if constexpr (SPLIT_B) {
            tma_load_3d(&tmB, &full[stage], sB, k0, tn * (BN / 2), g);
            tma_load_3d(&tmB, &full[stage], sB + (BN / 2) * 128, k0, p.f_half + tn * (BN / 2), g);
          } else if constexpr (!B_MN) {
            tma_load_3d(&tmB, &full[stage], sB, k0, tn * BN, g);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_3d(&tmB, &full[stage], sB + j * 8192, tn * BN + j * 64, k0, g);
          }
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // drain: every issued stage's bytes must have landed before the CTA exits
    long long n_wait = issued < STAGES ? issued : STAGES;
    int s = stage;
    uint32_t ph = phase;
    for (long long i = 0; i < n_wait; ++i) {
      if (--s < 0) {
        s = STAGES - 1;
        ph ^= 1;
      }
      mbar_wait(&full[s], ph, p.err, ERR_TIMEOUT_FULL);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t accphase = 0;
    bool ok = true, any = false;
    for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
      if (!mbar_wait(&accempty[acc], accphase ^ 1, p.err, ERR_TIMEOUT_TMEM_FREE)) break;
      tc_fence_after();
      const uint32_t dtm = tmem_base + acc * BN;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&full[stage], phase, p.err, ERR_TIMEOUT_FULL)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t aaddr = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t baddr = aaddr + L::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t ad, bd;
            if constexpr (!A_MN) ad = umma_smem_desc(aaddr + kk * 32, 16, 1024, kLayoutSW128);
            else ad = umma_smem_desc(aaddr + kk * 2048, 8192, 1024, kLayoutSW128);
            if constexpr (!B_MN) bd = umma_smem_desc(baddr + kk * 32, 16, 1024, kLayoutSW128);
            else bd = umma_smem_desc(baddr + kk * 2048, 8192, 1024, kLayoutSW128);
            umma_bf16(dtm, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          any = true;
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&accfull[acc]);
      __syncwarp();
      acc ^= 1;
      if (acc == 0) accphase ^= 1;
    }
    // drain: all issued MMAs complete before TMEM is released
    if (lane == 0 && any) {
      umma_commit(drain);
      mbar_wait(drain, 0, p.err, ERR_TIMEOUT_ACCUM);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..9)
    const int q = warp % 4;         // TMEM lane quarter this warp may access
    const int ch = (warp - 2) / 4;  // which column half of the tile
    int acc = 0;
    uint32_t accphase = 0, wphase = 0;
    EpiCtx ectx{smem + L::STG_OFF + (warp - 2) * STGW, STGW, &wbar[warp - 2], &wphase, &tmC, &tmX};
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      if (!mbar_wait(&accfull[acc], accphase, p.err, ERR_TIMEOUT_ACCUM)) break;
      tc_fence_after();
      const int g = t / tiles_per_g, r = t % tiles_per_g;
      const int tm = r / p.tiles_n, tn = r % p.tiles_n;
      const uint32_t tacc = tmem_base + acc * BN;
      uint8_t* stg = ectx.stg;
      if constexpr (EPI == EPI_LOGITS) {
        epilogue_logits<BN>(p, tacc, q, ch, lane, g, tm, tn, stg, &tmC);
      } else if constexpr (EPI != EPI_BF16) {
        if (p.tma_store) {
          if (!epilogue_tma<BN, EPI>(p, tacc, q, ch, lane, g, tm, tn, ectx)) break;
        } else {
          epilogue_tile<BN, EPI>(p, tacc, q, ch, lane, g, tm, tn, stg, &tmC);
        }
      } else {
        epilogue_tile<BN, EPI>(p, tacc, q, ch, lane, g, tm, tn, stg, &tmC);
      }
      tc_fence_before();
      mbar_arrive(&accempty[acc]);
      acc ^= 1;
      if (acc == 0) accphase ^= 1;
    }
    if (p.tma_store) {  // every staged store has landed before the CTA exits
      if (lane == 0) bulk_wait0();
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem_base, tmem_cols(BN));
}

// ============================================================== softmax-gradient operand
// One 64-element slab of dlogits in place: 8 x 16-byte chunks of bf16 logits at `row`
// (swizzled chunk order), element e of chunk j at index base + 8 j + e along the vocab.
// Same arithmetic as the CE kernel's pass 3 (ce_exp, RNE to bf16, label column minus sc).
ODP_DEVICE void xf_slab(uint8_t* row, int swz, float ob, float sc, int y, int base) {
  // all eight 16-byte loads first, then the 64 exponentials, then the stores: nothing
  // orders a load after an earlier store of the slab, so the chunks overlap
  uint4 v[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = *reinterpret_cast<const uint4*>(row + ((j ^ swz) << 4));
  const bool live = y >= 0;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = base + 8 * j + 2 * e;
      const float lo = ce_exp(__uint_as_float(w[e] << 16), ob);
      const float hi = ce_exp(__uint_as_float(w[e] & 0xffff0000u), ob);
      o[e] = pack_bf16(col == y ? lo - sc : lo, col + 1 == y ? hi - sc : hi);
    }
    v[j] = live ? make_uint4(o[0], o[1], o[2], o[3]) : make_uint4(0, 0, 0, 0);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) *reinterpret_cast<uint4*>(row + ((j ^ swz) << 4)) = v[j];
}

// Staging bytes per epilogue warp of the pair kernel: a 256-wide bf16 tile stages both of a
// warp's 32 x 64 boxes before one proxy fence and two TMA stores; other tiles one 4 KB box.
constexpr int stg2_bytes(int epi, int bn) { return (epi == EPI_BF16 && bn == 256) ? 8192 : 4096; }

// ============================================================== CTA-pair variant
// The same GEMM with each output tile (256 x BN) computed by a pair of CTAs on two SMs
// (cluster of 2, tcgen05.mma.cta_group::2): each CTA loads its own 128 rows of A and its
// own BN/2 rows of B, so every SM streams half as many bytes of B per FLOP as in the
// single-CTA kernel (the LM-head GEMMs are L2-bandwidth bound at 128 x 128). Loads are
// plain (never multicast) TMA copies into the issuing CTA's shared memory that complete
// on the leader CTA's mbarrier; the leader alone issues MMAs; commits arrive on both
// CTAs' barriers; each CTA's epilogue drains its own 128 TMEM lanes and the peer's
// epilogue warps release the accumulator on the leader's barrier remotely.
template <int BN, int STAGES, int STGW = 4096>
struct SmemLayout2 {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = (BN / 2) * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static_assert(STAGE_BYTES % 1024 == 0, "stages start on a swizzle-atom boundary");
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int STG_BYTES = 8 * STGW;  // STGW staging bytes per epilogue warp
  static constexpr int BAR_OFF = STG_OFF + STG_BYTES;
  static constexpr int TOTAL = BAR_OFF + 512 + 1024;
  static_assert(TOTAL <= 232448, "shared memory budget");
};

template <bool A_MN, bool B_MN, int BN, int STAGES, int EPI, int XF = 0>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(XF ? kThreadsXF : kThreads, 1)
    gemm2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                 const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmX, GemmParams p) {
  using L = SmemLayout2<BN, STAGES, stg2_bytes(EPI, BN)>;
  constexpr int HB = BN / 2;  // B rows held by each CTA
  // an MN-major B half that is not a whole number of 64-element 128-byte atoms (HB = 96)
  // is held as 32-element 64-byte-swizzled atoms
  constexpr bool B_SW64 = B_MN && (HB % 64) != 0;
  static_assert(!B_MN || HB % 32 == 0, "MN-major B half must be a multiple of 32");
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* accfull = empty + STAGES;
  uint64_t* accempty = accfull + 2;
  uint64_t* wbar = accempty + 2;  // one per epilogue warp: inputs of the TMA-store epilogue
  uint64_t* afull = wbar + 8;      // XF: this CTA's A tile of a stage has landed
  uint64_t* xdone = afull + STAGES;  // XF (leader): both CTAs' A tiles of a stage are transformed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(xdone + STAGES);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accfull[b], 1);
      mbar_init(&accempty[b], 16);  // one arrive per epilogue warp of both CTAs
    }
    for (int w = 0; w < 8; ++w) mbar_init(&wbar[w], 1);
    if constexpr (XF != 0) {
      for (int s = 0; s < STAGES; ++s) {
        mbar_init(&afull[s], 1);
        mbar_init(&xdone[s], 8);  // one arrival per transform warp of both CTAs
      }
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc_pair(tmem_holder, tmem_cols(BN));
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers are initialised before any remote signal
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  pdl_wait();     // global memory only from here on
  pdl_trigger();  // after this CTA's TMEM allocation
  const int tiles_per_g = p.tiles_m * p.tiles_n;
  constexpr uint32_t kIdesc = umma_idesc_bf16(2 * BM, BN, A_MN, B_MN);

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    const uint32_t full_leader = mapa_rank(&full[0], 0);
    int stage = 0;
    uint32_t phase = 0;
    long long issued = 0;
    bool ok = true;
    for (int t = pair; t < p.num_tiles && ok; t += npairs) {
      const int g = t / tiles_per_g, r = t % tiles_per_g;
      const int tm = r / p.tiles_n, tn = r % p.tiles_n;
      const int row0 = tm * 2 * BM + (int)rank * BM;
      const int col0 = tn * BN + (int)rank * HB;
      for (int kb = 0; kb < p.num_kb; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1, p.err, ERR_TIMEOUT_EMPTY)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          const uint32_t fb = full_leader + stage * 8;
          const int k0 = kb * BK;
          if constexpr (XF != 0) {
            // A lands on this CTA's own barrier (its transform warps rewrite it); the
            // leader's barrier counts only the B halves of both CTAs
            if (leader) mbar_expect_tx(&full[stage], 2 * L::B_BYTES);
            mbar_expect_tx(&afull[stage], L::A_BYTES);
            if constexpr (!A_MN) {
              tma_load_3d(&tmA, &afull[stage], sA, k0, row0, g);
            } else {
              tma_load_3d(&tmA, &afull[stage], sA, row0, k0, g);
              tma_load_3d(&tmA, &afull[stage], sA + 8192, row0 + 64, k0, g);
            }
          } else {
            if (leader) mbar_expect_tx(&full[stage], 2 * L::STAGE_BYTES);
            if constexpr (!A_MN) {
              tma_load_3d_pair(&tmA, fb, sA, k0, row0, g);
            } else {
              tma_load_3d_pair(&tmA, fb, sA, row0, k0, g);
              tma_load_3d_pair(&tmA, fb, sA + 8192, row0 + 64, k0, g);
            }
          }
          if constexpr (!B_MN) {
            tma_load_3d_pair(&tmB, fb, sB, k0, col0, g);
          } else if constexpr (B_SW64) {
#pragma unroll
            for (int j = 0; j < HB / 32; ++j) tma_load_3d_pair(&tmB, fb, sB + j * 4096, col0 + j * 32, k0, g);
          } else {
#pragma unroll
            for (int j = 0; j < HB / 64; ++j) tma_load_3d_pair(&tmB, fb, sB + j * 8192, col0 + j * 64, k0, g);
          }
        }
        __syncwarp();
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
    // drain: the MMA has consumed (so the copies have landed in) every stage filled here
    long long n_wait = issued < STAGES ? issued : STAGES;
    int s = stage;
    uint32_t ph = phase;
    for (long long i = 0; i < n_wait; ++i) {
      if (--s < 0) {
        s = STAGES - 1;
        ph ^= 1;
      }
      mbar_wait(&empty[s], ph, p.err, ERR_TIMEOUT_EMPTY);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t accphase = 0;
      bool ok = true;
      for (int t = pair; t < p.num_tiles && ok; t += npairs) {
        if (!mbar_wait(&accempty[acc], accphase ^ 1, p.err, ERR_TIMEOUT_TMEM_FREE)) break;
        tc_fence_after();
        const uint32_t dtm = tmem_base + acc * BN;
        for (int kb = 0; kb < p.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, p.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          if constexpr (XF != 0) {
            if (!mbar_wait_cluster(&xdone[stage], phase, p.err, ERR_TIMEOUT_FULL)) {
              ok = false;
              break;
            }
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t aaddr = smem_u32(smem + stage * L::STAGE_BYTES);
            const uint32_t baddr = aaddr + L::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              uint64_t ad, bd;
              if constexpr (!A_MN) ad = umma_smem_desc(aaddr + kk * 32, 16, 1024, kLayoutSW128);
              else ad = umma_smem_desc(aaddr + kk * 2048, 8192, 1024, kLayoutSW128);
              if constexpr (!B_MN) bd = umma_smem_desc(baddr + kk * 32, 16, 1024, kLayoutSW128);
              else if constexpr (B_SW64) bd = umma_smem_desc(baddr + kk * 1024, 4096, 512, kLayoutSW64);
              else bd = umma_smem_desc(baddr + kk * 2048, 8192, 1024, kLayoutSW128);
              umma_bf16_pair(dtm, ad, bd, kIdesc, (kb | kk) != 0 ? 1u : 0u);
            }
            umma_commit_pair(&empty[stage]);
          }
          __syncwarp();
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        if (lane == 0) umma_commit_pair(&accfull[acc]);
        __syncwarp();
        acc ^= 1;
        if (acc == 0) accphase ^= 1;
      }
    }
  } else if (XF != 0 && warp >= 10) {
    // ------------------------------------------------------------ A transform (both CTAs)
    // logits -> dlogits in shared memory, then one arrival per warp on the leader's xdone
    // barrier (shared-memory writes fenced to the async proxy first). Two groups of four
    // warps take alternate stages, so one group's waits and fences overlap the other's
    // arithmetic.
    const int grp = (warp - 10) / 4;
    const int tid = ((warp - 10) % 4) * 32 + lane;  // 0..127 within the group
    const uint32_t xdone_leader = mapa_rank(&xdone[0], 0);
    int stage = 0;
    uint32_t phase = 0;
    long long it = 0;  // stage uses so far (both groups' share)
    bool ok = true;
    for (int t = pair; t < p.num_tiles && ok; t += npairs) {
      const int gg = t / tiles_per_g, r = t % tiles_per_g;
      const int tm = r / p.tiles_n;
      const int path = gg / p.xf_split;
      const long long tok0 = (long long)(gg % p.xf_split) * p.K;  // token offset of this split
      const long long rbase = path * p.xf_ms + tok0;
      const float sc = p.xf_sc[path];
      const int row0 = tm * 2 * BM + (int)rank * BM;
      // (label, ob) of this thread's token: XF 1 one per tile (row tid of A); XF 2 one per
      // k-block (token row kb * 64 + tid % 64), fetched one own-stage ahead
      auto fetch = [&](long long tok, long long lim, int& y, float& ob) {
        y = -1;
        ob = 0.f;
        if (tok < lim) {
          y = p.xf_lab[rbase + tok];
          ob = p.xf_ob[rbase + tok];
        }
      };
      int y, yn;
      float ob, obn;
      const int k = tid & 63, h = tid >> 6;
      if (XF == 1) fetch(row0 + tid, p.M, y, ob);
      const int kb0 = (int)((grp - (it & 1) + 2) & 1);  // this group's first k-block of the tile
      if (XF == 2) fetch((long long)kb0 * BK + k, p.K, yn, obn);
      for (int kb = 0; kb < p.num_kb; ++kb, ++it) {
        if ((it & 1) == grp) {
          if (!mbar_wait(&afull[stage], phase, p.err, ERR_TIMEOUT_FULL)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          if constexpr (XF == 1) {
            // K-major: row tid holds vocab columns [kb * 64, kb * 64 + 64) of token row0 + tid
            xf_slab(sA + tid * 128, tid & 7, ob, sc, y, kb * BK);
          } else {
            // MN-major: 64 token rows x (two 64-vocab halves); thread = (token k, half h)
            y = yn;
            ob = obn;
            fetch((long long)(kb + 2) * BK + k, kb + 2 < p.num_kb ? p.K : 0, yn, obn);
            xf_slab(sA + h * 8192 + k * 128, k & 7, ob, sc, y, row0 + h * 64);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(xdone_leader + stage * 8);
          __syncwarp();
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp % 4;
    const int ch = (warp - 2) / 4;
    const uint32_t accempty_leader = mapa_rank(&accempty[0], 0);
    constexpr int STGW = stg2_bytes(EPI, BN);
    uint8_t* stg = smem + L::STG_OFF + (warp - 2) * STGW;
    int acc = 0;
    uint32_t accphase = 0, wphase = 0;
    EpiCtx ectx{stg, 4096, &wbar[warp - 2], &wphase, &tmC, &tmX};
    for (int t = pair; t < p.num_tiles; t += npairs) {
      if (!mbar_wait(&accfull[acc], accphase, p.err, ERR_TIMEOUT_ACCUM)) break;
      tc_fence_after();
      const int g = t / tiles_per_g, r = t % tiles_per_g;
      const int tm = r / p.tiles_n, tn = r % p.tiles_n;
      // this CTA holds rows [tm * 256 + rank * 128, +128) of the pair tile: a 128-row tile index
      bool ok = true;
      if constexpr (EPI == EPI_F32) {
        if (p.tma_store) ok = epilogue_tma<BN, EPI>(p, tmem_base + acc * BN, q, ch, lane, g, tm * 2 + (int)rank, tn, ectx);
        else epilogue_tile<BN, EPI, STGW>(p, tmem_base + acc * BN, q, ch, lane, g, tm * 2 + (int)rank, tn, stg, &tmC);
      } else {
        epilogue_tile<BN, EPI, STGW>(p, tmem_base + acc * BN, q, ch, lane, g, tm * 2 + (int)rank, tn, stg, &tmC);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(accempty_leader + acc * 8);
      __syncwarp();
      if (!ok) break;
      acc ^= 1;
      if (acc == 0) accphase ^= 1;
    }
    if (p.tma_store) {
      if (lane == 0) bulk_wait0();
      __syncwarp();
    }
  }

  tc_fence_before();
  cluster_sync();  // every MMA consumed, every remote arrival delivered, before TMEM goes away
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem_base, tmem_cols(BN));
}

// ============================================================== host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// bf16 3-D map: x = contiguous dim (extent inner), y = rows (extent outer, stride ld),
// z = group (extent G, stride sg). Box = {64, box_rows, 1}, 128-byte swizzle.
static CUtensorMap make_map(const void* base, long long inner, long long outer, long long ld, int G,
                            long long sg, int box_rows, int box_inner = 64,
                            CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B,
                            CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, int esz = 2) {
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * esz) % 16 == 0, "row stride must be a multiple of 16 bytes");
  TORCH_CHECK(G == 1 || (sg * esz) % 16 == 0, "group stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)outer, (cuuint64_t)G};
  long long gstride = G > 1 ? sg * esz : ((outer * ld * esz + 15) / 16) * 16;
  cuuint64_t strides[2] = {(cuuint64_t)(ld * esz), (cuuint64_t)gstride};
  cuuint32_t box[3] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = get_encode()(&m, dt, 3, const_cast<void*>(base), dims, strides, box, es,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

static bool al16(const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; }

// Output (and epilogue-input) maps of the TMA-store epilogues of fp32 / residual / SwiGLU
// outputs; false when a base, row stride or group stride is not 16-byte aligned (those
// calls keep the per-thread stores).
template <int EPI>
static bool out_maps(const GemmParams& p, CUtensorMap& mc, CUtensorMap& mx) {
  if (getenv("ODP_GEMM_NO_TMA_STORE")) return false;
  const auto F32 = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const auto B16 = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  if constexpr (EPI == EPI_F32 || EPI == EPI_RESID) {
    if (!al16(p.C) || (p.ldc * 4) % 16 || (p.G > 1 && (p.sc * 4) % 16)) return false;
    mc = make_map(p.C, p.N, p.M, p.ldc, p.G, p.sc, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, F32, 4);
    if constexpr (EPI == EPI_RESID) {
      if (!al16(p.R) || (p.ldr * 4) % 16 || (p.G > 1 && (p.sr * 4) % 16)) return false;
      mx = make_map(p.R, p.N, p.M, p.ldr, p.G, p.sr, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, F32, 4);
    } else {
      mx = mc;
    }
    return true;
  } else if constexpr (EPI == EPI_SWIGLU || EPI == EPI_SWIGLU_BWD) {
    const long long F = p.f_half;
    if (F % 32 || !al16(p.C) || !al16(p.aux) || (p.ldc * 2) % 16 || (p.ldx * 2) % 16 ||
        (p.G > 1 && ((p.sc * 2) % 16 || (p.sx * 2) % 16)))
      return false;
    // SwiGLU: C = H [M, F], aux = [g | u] [M, 2F]; backward: C = [dG | dU] [M, 2F], aux = [g | u]
    const long long c_inner = EPI == EPI_SWIGLU ? F : 2 * F;
    if (EPI == EPI_SWIGLU_BWD && p.N > F) return false;
    mc = make_map(p.C, c_inner, p.M, p.ldc, p.G, p.sc, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B, B16, 2);
    mx = make_map(p.aux, 2 * F, p.M, p.ldx, p.G, p.sx, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B, B16, 2);
    return true;
  } else {
    return false;
  }
}

template <bool A_MN, bool B_MN, int BN, int STAGES, int EPI>
static void launch_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mx,
                     GemmParams& p, cudaStream_t st, int max_ctas) {
  using L = SmemLayout<BN, STAGES, stg_warp_bytes(EPI, false)>;
  auto kern = gemm_kernel<A_MN, B_MN, BN, STAGES, EPI>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
    attr_set = true;
  }
  int grid = std::min(p.num_tiles, max_ctas > 0 ? max_ctas : num_sms());
  C10_CUDA_CHECK(odp::launch_pdl(kern, dim3(grid), dim3(kThreads), L::TOTAL, st, ma, mb, mc, mx, p));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <bool A_MN, bool B_MN, int BN, int STAGES, int EPI, int XF = 0>
static void launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const CUtensorMap& mx,
                        GemmParams& p, cudaStream_t st, int max_ctas) {
  using L = SmemLayout2<BN, STAGES, stg2_bytes(EPI, BN)>;
  auto kern = gemm2_kernel<A_MN, B_MN, BN, STAGES, EPI, XF>;
  static bool attr_set = false;
  if (!attr_set) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr_set = true;
  }
  int grid = std::min(2 * p.num_tiles, max_ctas > 0 ? max_ctas : num_sms());
  grid &= ~1;  // whole CTA pairs
  C10_CUDA_CHECK(odp::launch_pdl(kern, dim3(grid), dim3(XF ? kThreadsXF : kThreads), L::TOTAL, st, ma, mb, mc, mx, p));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Operand description: data pointer, leading dim (elements), group stride (elements).
struct Operand {
  const void* ptr;
  long long ld, sg;
  bool mn;  // true: stored [K, rows] (rows contiguous); false: stored [rows, K]
};

// Which (epilogue, operand majors, tile width) combinations are instantiated.
template <int EPI, bool AM, bool BMN, int BN>
constexpr bool cfg_ok() {
  if (EPI == EPI_SWIGLU || EPI == EPI_LOGITS) return !AM && !BMN && BN == 128;
  if (EPI == EPI_SWIGLU_BWD) return !AM && BMN && BN != 256;
  if (EPI == EPI_RESID || EPI == EPI_BF16) return !AM && BN != 256 && BN != 192;
  // 192-wide tiles (N = 384 in two tiles): fp32 outputs of long-K products such as the
  // LM-head input and weight gradients
  if (BN == 192) return EPI == EPI_F32;
  return BN != 256 || (!AM && !BMN);
}

template <int EPI, bool AM, bool BMN, int BN>
constexpr bool cfg2_ok() {
  if (BN == 192) return EPI == EPI_F32;
  if (EPI == EPI_BF16) return !AM;
  return EPI == EPI_F32;
}

// CTA-pair path: bf16 / fp32 epilogues with at least one full 256-row pair tile.
template <int EPI>
static bool dispatch_pair(const Operand& A, const Operand& B, GemmParams& p, cudaStream_t st, int max_ctas) {
  if constexpr (EPI != EPI_BF16 && EPI != EPI_F32) {
    return false;
  } else {
    const char* env = getenv("ODP_GEMM_2SM");
    if ((env && env[0] == '0') || p.M < 2 * BM || (max_ctas > 0 && max_ctas < 2)) return false;
    if (EPI == EPI_BF16 && A.mn) return false;
    // 256-wide pair tiles for wide outputs; 192-wide pair tiles (each CTA holds 96 columns
    // of B) for fp32 outputs whose width is a multiple of 192 but not of 256 (N = 384: the
    // input and weight gradients of hidden-384 layers and LM heads). 128-wide pair tiles
    // measured no faster than the single-CTA kernel.
    const bool w256 = p.N >= 256 && (p.N % 256 == 0 || p.N >= 2048);
    const bool w192 = EPI == EPI_F32 && !w256 && p.N % 192 == 0;
    if (!w256 && !w192) return false;
    const int bn = w256 ? 256 : 192;
    p.tiles_m = (p.M + 2 * BM - 1) / (2 * BM);
    p.tiles_n = (p.N + bn - 1) / bn;
    p.num_tiles = p.tiles_m * p.tiles_n * p.G;
    CUtensorMap ma = A.mn ? make_map(A.ptr, p.M, p.K, A.ld, p.G, A.sg, 64) : make_map(A.ptr, p.K, p.M, A.ld, p.G, A.sg, BM);
    CUtensorMap mb = !B.mn ? make_map(B.ptr, p.K, p.N, B.ld, p.G, B.sg, bn / 2)
                     : (bn / 2) % 64 ? make_map(B.ptr, p.N, p.K, B.ld, p.G, B.sg, 64, 32, CU_TENSOR_MAP_SWIZZLE_64B)
                                     : make_map(B.ptr, p.N, p.K, B.ld, p.G, B.sg, 64);
    CUtensorMap mc = ma, mx = ma;
    bool tma_ok;
    if constexpr (EPI == EPI_BF16) {
      tma_ok = al16(p.C) && (p.ldc * 2) % 16 == 0 && (p.G == 1 || (p.sc * 2) % 16 == 0) &&
               !getenv("ODP_GEMM_NO_TMA_STORE");
      if (tma_ok) mc = make_map(p.C, p.N, p.M, p.ldc, p.G, p.sc, 32);
    } else {
      tma_ok = out_maps<EPI>(p, mc, mx);
    }
    TORCH_CHECK(tma_ok || !p.sqp, "gemm: box sums of squares need a TMA-storable fp32 output");
    p.tma_store = tma_ok ? 1 : 0;
    if constexpr (EPI == EPI_F32) {
      if (p.xf) {
        // softmax-gradient operand: the LM-head input gradient (A K-major, B MN-major) and
        // weight gradient (both MN-major)
        TORCH_CHECK((p.xf == 1 && !A.mn && B.mn) || (p.xf == 2 && A.mn && B.mn),
                    "gemm_ce_grad: unsupported operand layout");
#define ODP_GOX(AM, BNV, ST, X)                                                                          \
  if (A.mn == AM && bn == BNV && p.xf == X) {                                                            \
    launch_pair<AM, true, BNV, fit_stages((BM + BNV / 2) * BK * 2, 8 * stg2_bytes(EPI, BNV), ST), EPI, X>(ma, mb, mc, mx, p, \
                                                                                        st, max_ctas);   \
    return true;                                                                                         \
  }
        ODP_GOX(false, 256, 6, 1)
        ODP_GOX(false, 192, 7, 1)
        ODP_GOX(true, 256, 6, 2)
        ODP_GOX(true, 192, 7, 2)
#undef ODP_GOX
        return false;
      }
    }
#define ODP_GO2(AM, BMN, BNV, ST)                                                                        \
  if constexpr (cfg2_ok<EPI, AM, BMN, BNV>()) {                                                          \
    if (A.mn == AM && B.mn == BMN && bn == BNV) {                                                        \
      launch_pair<AM, BMN, BNV, fit_stages((BM + BNV / 2) * BK * 2, 8 * stg2_bytes(EPI, BNV), ST), EPI>(ma, mb, mc, mx, p, \
                                                                                        st, max_ctas);   \
      return true;                                                                                       \
    }                                                                                                    \
  }
    ODP_GO2(false, false, 256, 6)
    ODP_GO2(false, true, 256, 6)
    ODP_GO2(true, false, 256, 6)
    ODP_GO2(true, true, 256, 6)
    ODP_GO2(false, false, 192, 7)
    ODP_GO2(false, true, 192, 7)
    ODP_GO2(true, false, 192, 7)
    ODP_GO2(true, true, 192, 7)
#undef ODP_GO2
    return false;
  }
}

template <int EPI>
static void dispatch(const Operand& A, const Operand& B, GemmParams& p, int bn, cudaStream_t st, int max_ctas) {
  if (dispatch_pair<EPI>(A, B, p, st, max_ctas)) return;
  TORCH_CHECK(!p.xf, "gemm_ce_grad: needs the CTA-pair kernel (M >= 256 and N a multiple of 192 or 256)");
  const int rowsB = EPI == EPI_SWIGLU ? bn / 2 : bn;
  CUtensorMap ma = A.mn ? make_map(A.ptr, p.M, p.K, A.ld, p.G, A.sg, 64) : make_map(A.ptr, p.K, p.M, A.ld, p.G, A.sg, BM);
  long long b_rows_extent = EPI == EPI_SWIGLU ? 2LL * p.f_half : p.N;
  CUtensorMap mb = B.mn ? make_map(B.ptr, p.N, p.K, B.ld, p.G, B.sg, 64)
                        : make_map(B.ptr, p.K, b_rows_extent, B.ld, p.G, B.sg, rowsB);
  // bf16 outputs of 128-wide tiles, and fp32 / residual / SwiGLU outputs of any tile
  // width, leave through TMA stores when the layout allows it
  CUtensorMap mc = ma, mx = ma;
  bool tma_ok;
  if constexpr (EPI == EPI_BF16 || EPI == EPI_LOGITS) {
    tma_ok = bn == 128 && al16(p.C) && (p.ldc * 2) % 16 == 0 && (p.G == 1 || (p.sc * 2) % 16 == 0) &&
             !getenv("ODP_GEMM_NO_TMA_STORE");
    if (tma_ok) mc = make_map(p.C, p.N, p.M, p.ldc, p.G, p.sc, 32);
  } else {
    tma_ok = out_maps<EPI>(p, mc, mx);
  }
  TORCH_CHECK(tma_ok || !p.sqp, "gemm: box sums of squares need a TMA-storable fp32 output");
  p.tma_store = tma_ok ? 1 : 0;
#define ODP_GO(AM, BMN, BNV, ST)                                                                       \
  if constexpr (cfg_ok<EPI, AM, BMN, BNV>()) {                                                         \
    if (A.mn == AM && B.mn == BMN && bn == BNV) {                                                      \
      launch_t<AM, BMN, BNV, fit_stages((BM + BNV) * BK * 2, 8 * stg_warp_bytes(EPI, false), ST), EPI>( \
          ma, mb, mc, mx, p, st, max_ctas);                                                            \
      return;                                                                                          \
    }                                                                                                  \
  }
  ODP_GO(false, false, 128, 6)
  ODP_GO(false, true, 128, 6)
  ODP_GO(true, false, 128, 6)
  ODP_GO(true, true, 128, 6)
  ODP_GO(false, false, 64, 8)
  ODP_GO(false, true, 64, 8)
  ODP_GO(true, false, 64, 8)
  ODP_GO(true, true, 64, 8)
  ODP_GO(false, false, 256, 4)
  ODP_GO(false, false, 192, 4)
  ODP_GO(false, true, 192, 4)
  ODP_GO(true, false, 192, 4)
  ODP_GO(true, true, 192, 4)
#undef ODP_GO
  TORCH_CHECK(false, "unsupported GEMM configuration");
}

}  // namespace odp

namespace odp {

// ---------------------------------------------------------------- split-K reduction
// A weight-gradient GEMM whose output tiles cannot fill the GPU runs as S times as many
// groups over K / S each (for these operands group g's K rows start at g * K * ld, so the
// splits are plain groups of the same GEMM): ws[g * S + s] holds split s of group g.
// C[g] = sum_s ws[g * S + s] (+ beta * C) in split order, and, if sqp is given, the sum of
// squares of every 32 x 32 box of C at sqp[g * sq_ld + (row / 32) * ceil(N / 32) + col / 32].
// One 256-thread block per 32 x 32 box: 32 rows x 8 threads x 4 columns.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, int S, int M, int N,
                                                            float* __restrict__ C, long long ldc, long long sc,
                                                            float* __restrict__ sqp, long long sq_ld, float beta) {
  pdl_wait();
  pdl_trigger();
  const int nbc = (N + 31) / 32, nbr = (M + 31) / 32;
  const int g = blockIdx.y, br = blockIdx.x / nbc, bc = blockIdx.x % nbc;
  const int r = br * 32 + threadIdx.x / 8, c = bc * 32 + (threadIdx.x % 8) * 4;
  float q = 0.f;
  if (r < M && c < N) {
    const long long mn = (long long)M * N;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    const int n = min(4, N - c);
    const float* w0 = ws + (long long)g * S * mn + (long long)r * N + c;
    if (n == 4 && (N % 4) == 0 && S <= 8) {
      // every split's load in flight at once, then the sum in split order
      float4 x[8];
#pragma unroll
      for (int sp = 0; sp < 8; ++sp)
        if (sp < S) x[sp] = *reinterpret_cast<const float4*>(w0 + sp * mn);
#pragma unroll
      for (int sp = 0; sp < 8; ++sp)
        if (sp < S) {
          v[0] += x[sp].x;
          v[1] += x[sp].y;
          v[2] += x[sp].z;
          v[3] += x[sp].w;
        }
    } else {
      for (int sp = 0; sp < S; ++sp)
        for (int i = 0; i < n; ++i) v[i] += w0[sp * mn + i];
    }
    float* dst = C + g * sc + (long long)r * ldc + c;
    for (int i = 0; i < n; ++i) {
      const float o = beta != 0.f ? v[i] + beta * dst[i] : v[i];
      dst[i] = o;
      q = fmaf(o, o, q);
    }
  }
  if (sqp) {
    q = warp_sum(q);
    __shared__ float red[8];
    if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = q;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int w = 0; w < 8; ++w) t += red[w];
      sqp[(long long)g * sq_ld + (long long)br * nbc + bc] = t;
    }
  }
  (void)nbr;
}

}  // namespace odp

// ---------------------------------------------------------------- torch entry
// A: tensor whose storage holds G groups; a_mn selects its major; shapes are given
// explicitly so callers can pass views into flat parameter buffers.
void gemm_bf16(torch::Tensor A, int64_t lda, int64_t sa, bool a_mn, torch::Tensor B, int64_t ldb, int64_t sb,
               bool b_mn, torch::Tensor C, int64_t ldc, int64_t sc, int64_t M, int64_t N, int64_t K, int64_t G,
               int64_t epi, int64_t bn, c10::optional<torch::Tensor> R, int64_t ldr, int64_t sr,
               c10::optional<torch::Tensor> aux, int64_t ldx, int64_t sx, c10::optional<torch::Tensor> part,
               double beta, int64_t f_half, torch::Tensor err, int64_t max_ctas,
               c10::optional<torch::Tensor> sq_part, int64_t sq_ld) {
  using namespace odp;
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands");
  c10::cuda::CUDAGuard guard(A.device());
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.G = (int)G;
  p.f_half = (int)f_half;
  const int tile_n = (epi == EPI_SWIGLU) ? (int)bn / 2 : (int)bn;
  p.tiles_m = (int)((M + BM - 1) / BM);
  p.tiles_n = (int)(((epi == EPI_SWIGLU ? f_half : N) + tile_n - 1) / tile_n);
  p.num_tiles = p.tiles_m * p.tiles_n * (int)G;
  p.num_kb = (int)((K + BK - 1) / BK);
  p.C = C.data_ptr();
  p.ldc = ldc;
  p.sc = sc;
  p.R = R.has_value() ? R->data_ptr<float>() : nullptr;
  p.ldr = ldr;
  p.sr = sr;
  p.aux = aux.has_value() ? aux->data_ptr() : nullptr;
  p.ldx = ldx;
  p.sx = sx;
  p.part = part.has_value() ? part->data_ptr<float>() : nullptr;
  p.sqp = sq_part.has_value() ? sq_part->data_ptr<float>() : nullptr;
  p.sq_ld = sq_ld;
  TORCH_CHECK(!p.sqp || epi == EPI_F32, "gemm: box sums of squares are produced by the fp32 epilogue only");
  p.beta = (float)beta;
  p.err = err.data_ptr<int>();
  Operand a{A.data_ptr(), lda, sa, a_mn}, b{B.data_ptr(), ldb, sb, b_mn};
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  switch (epi) {
    case EPI_BF16: dispatch<EPI_BF16>(a, b, p, (int)bn, st, (int)max_ctas); break;
    case EPI_F32: dispatch<EPI_F32>(a, b, p, (int)bn, st, (int)max_ctas); break;
    case EPI_RESID: dispatch<EPI_RESID>(a, b, p, (int)bn, st, (int)max_ctas); break;
    case EPI_SWIGLU: dispatch<EPI_SWIGLU>(a, b, p, (int)bn, st, (int)max_ctas); break;
    case EPI_SWIGLU_BWD: dispatch<EPI_SWIGLU_BWD>(a, b, p, (int)bn, st, (int)max_ctas); break;
    case EPI_LOGITS: dispatch<EPI_LOGITS>(a, b, p, (int)bn, st, (int)max_ctas); break;
    default: TORCH_CHECK(false, "unknown epilogue ", epi);
  }
}

// fp32 GEMM whose A operand is bf16 logits turned into the cross-entropy dlogits on the fly
// (the CE kernel's stats-only form wrote ob per token): xf = 1 for the LM-head input
// gradient (A = logits [tokens, vocab], K-major), xf = 2 for its weight gradient (A =
// logits^T, MN-major, K = tokens, optionally split over K into xf_split parts that run as
// G * xf_split groups). ob / labels: [paths][ms] with the token rows this GEMM sees at
// offset 0; sc: [paths] (1 / valid labels). The logits are only read.
void gemm_ce_grad(torch::Tensor A, int64_t lda, int64_t sa, bool a_mn, torch::Tensor B, int64_t ldb, int64_t sb,
                  bool b_mn, torch::Tensor C, int64_t ldc, int64_t sc, int64_t M, int64_t N, int64_t K, int64_t G,
                  double beta, torch::Tensor err, c10::optional<torch::Tensor> sq_part, int64_t sq_ld, int64_t xf,
                  torch::Tensor ob, torch::Tensor labels, torch::Tensor scale, int64_t ms, int64_t split) {
  using namespace odp;
  TORCH_CHECK(A.is_cuda() && B.is_cuda() && C.is_cuda(), "gemm_ce_grad: CUDA tensors required");
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm_ce_grad: bf16 operands");
  TORCH_CHECK(xf == 1 || xf == 2, "gemm_ce_grad: xf is 1 (input gradient) or 2 (weight gradient)");
  TORCH_CHECK(ob.scalar_type() == at::kFloat && labels.scalar_type() == at::kInt && scale.scalar_type() == at::kFloat,
              "gemm_ce_grad: fp32 ob / scale, int32 labels");
  TORCH_CHECK(split >= 1 && G % split == 0, "gemm_ce_grad: G must be a multiple of split");
  c10::cuda::CUDAGuard guard(A.device());
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.G = (int)G;
  p.num_kb = (int)((K + BK - 1) / BK);
  p.C = C.data_ptr();
  p.ldc = ldc;
  p.sc = sc;
  p.sqp = sq_part.has_value() ? sq_part->data_ptr<float>() : nullptr;
  p.sq_ld = sq_ld;
  p.beta = (float)beta;
  p.err = err.data_ptr<int>();
  p.xf = (int)xf;
  p.xf_ob = ob.data_ptr<float>();
  p.xf_lab = labels.data_ptr<int>();
  p.xf_sc = scale.data_ptr<float>();
  p.xf_ms = ms;
  p.xf_split = (int)split;
  Operand a{A.data_ptr(), lda, sa, a_mn}, b{B.data_ptr(), ldb, sb, b_mn};
  dispatch<EPI_F32>(a, b, p, 192, at::cuda::getCurrentCUDAStream(), 0);
}

// ws: [G * S][M][N] fp32 split partials (group-major); C: G groups of [M][N] at (ldc, sc).
void gemm_splitk_reduce(torch::Tensor ws, int64_t S, int64_t G, int64_t M, int64_t N, torch::Tensor C, int64_t ldc,
                        int64_t sc, c10::optional<torch::Tensor> sq_part, int64_t sq_ld, double beta) {
  c10::cuda::CUDAGuard guard(ws.device());
  TORCH_CHECK(ws.numel() >= G * S * M * N, "gemm_splitk_reduce: workspace too small");
  dim3 grid((unsigned)(((M + 31) / 32) * ((N + 31) / 32)), (unsigned)G);
  C10_CUDA_CHECK(odp::launch_pdl(odp::splitk_reduce_kernel, grid, dim3(256), 0, at::cuda::getCurrentCUDAStream(),
                                 ws.data_ptr<float>(), (int)S, (int)M, (int)N, C.data_ptr<float>(), ldc, sc,
                                 sq_part.has_value() ? sq_part->data_ptr<float>() : nullptr, sq_ld,
                                 (float)beta));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
