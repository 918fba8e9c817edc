// Causal self-attention on the 5th-generation tensor cores (tcgen05 + TMEM) for
// sequences of at most 128 tokens, head_dim 64, GQA, reading q/k/v straight out of the
// fused QKV projection output [GB, S, (nh + 2 nkv) * 64] (bf16) with RoPE applied while
// the tiles are staged (same rounding points as the mma.sync kernels in attention.cu).
//
// A whole (sequence, head) is one 128-row tile, so each CTA does the entire attention
// of one head with single-tile MMAs (M = 128):
//
// forward, one CTA per (head, sequence), 128 threads, thread t owns query row t:
//   S = Q K^T            -> TMEM columns [0, 128)       (4 MMAs, K = 64)
//   row softmax in registers from tcgen05.ld (no cross-thread reduction), P in bf16
//   written to shared memory over the Q/K tiles (both dead once S is done)
//   O = P V              -> TMEM columns [0, 64)        (8 MMAs, K = 128)
//   48 KB shared memory and 128 TMEM columns: four CTAs per SM.
//
// backward, one CTA per (kv head, sequence), 256 threads, looping over the query heads
// of the kv group (dK, dV accumulate in TMEM across them):
//   S = Q K^T -> [0,128), dP = dO V^T -> [128,256)
//   P = exp2(S * scale * log2e - lse * log2e), dS = P (dP - delta) with delta = rowsum(dO O)
//   computed in the kernel; P and dS stored once in shared memory as [query][key] tiles,
//   read K-major for dQ = dS K and MN-major (as P^T, dS^T) for
//   dV += P^T dO -> [256,320), dK += dS^T Q -> [320,384), dQ = dS K -> [384,448)
//   scale and the transpose of RoPE are applied in the epilogues.
// When every kv head serves one query head (no accumulation across heads), a lean variant
// uses 256 TMEM columns and 96 KB of shared memory so that two CTAs share an SM: dV goes
// into S's columns and dK, dQ into [64,128) and dP's [128,192) once S and dP are read
// out; P and dS share one pair of tiles (dV = P^T dO is issued and completed before dS,
// kept in registers meanwhile, overwrites P).
//
// Operand tiles are [128 rows][64 bf16] in the canonical 128-byte-swizzle layout (16-byte
// chunk index XOR row % 8, 8-row groups 1024 bytes apart), written by the threads
// themselves (RoPE has to be applied on the way in), then published to the tensor core
// with fence.proxy.async. One elected thread issues every MMA; completion is signalled
// through tcgen05.commit on an mbarrier whose waits are bounded (error word, no hang).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {
namespace attn_tc {

constexpr int D = 64;
constexpr int T = 128;               // rows of a tile = maximum sequence length
constexpr int TILE = T * 128;        // bytes of one [128][64] bf16 tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kFwdSmem = 3 * TILE + 1024;
constexpr int kBwdSmem = 8 * TILE + 1024;
constexpr int kBwdSmemLean = 6 * TILE + 1024;

struct Args {
  const __nv_bfloat16* qkv;
  long long ld;  // (nh + 2 nkv) * 64
  int S, nh, nkv;
  const float* cosT;
  const float* sinT;
  __nv_bfloat16* o;  // [GB, S, nh * 64]
  long long ldo;
  float* lse;        // [GB, nh, S] natural-log log-sum-exp of the scaled scores
  const __nv_bfloat16* dout;
  __nv_bfloat16* dqkv;
  float* delta;      // [GB, nh, S] rowsum(dO o), written by the flash dQ kernel
  float scale;
  int* err;
  // flash kernels: q|k with RoPE already applied ([GB, S, (nh + nkv) * 64], row stride ldr),
  // written once per call by rope_qk_kernel; null = rotate each staged tile instead
  const __nv_bfloat16* qkr;
  long long ldr;
};

// bf16 round-to-nearest-even on the integer pipe: add 0x7FFF plus the lowest kept bit and
// keep the high half. Identical to cvt.rn.bf16 for every finite value and infinity (a NaN
// with a payload only in the low 16 bits would become infinity; none arise here). This
// kernel packs about as many values as it multiplies, and the conversion unit, not the
// tensor core or HBM, bounded it; this form runs on the far wider integer ALUs. It hides
// the common pack_bf16 inside this namespace.
ODP_DEVICE uint32_t bf16_rne_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return u + 0x7FFFu + ((u >> 16) & 1u);
}
ODP_DEVICE uint32_t pack_bf16(float lo, float hi) {
  return __byte_perm(bf16_rne_bits(lo), bf16_rne_bits(hi), 0x7632);
}

// The hardware base-2 exponential (ex2.approx, flush-to-zero): the softmax probabilities
// are rounded to bf16 right after, far coarser than its error.
ODP_DEVICE float ex2_fast(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

ODP_DEVICE uint32_t sw_off(int row, int col) {
  return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2);
}

ODP_DEVICE void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// K-major operand: a [128 rows][64] tile, k-step kk covers columns [16 kk, 16 kk + 16).
ODP_DEVICE uint64_t desc_k(uint32_t tile, int kk) { return umma_smem_desc(tile + kk * 32, 16, 1024, kLayoutSW128); }
// MN-major operand: rows are the K index, k-step kk covers rows [16 kk, 16 kk + 16);
// consecutive 64-wide M/N chunks are separate tiles TILE bytes apart.
ODP_DEVICE uint64_t desc_mn(uint32_t tile, int kk) {
  return umma_smem_desc(tile + kk * 2048, TILE, 1024, kLayoutSW128);
}

ODP_DEVICE uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

ODP_DEVICE void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
ODP_DEVICE void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// Start copying rows [0, 128) of 64 columns at col0 of a [S, ld] bf16 matrix into a
// swizzled tile with cp.async (every copy of every tile in flight at once); rows >= S
// are zero-filled. Complete with cp_async_wait_all + a barrier.
template <int NT>
ODP_DEVICE void stage_async(uint8_t* tile, const __nv_bfloat16* src, long long ld, int col0, int S) {
  for (int i = threadIdx.x; i < T * 8; i += NT) {
    const int r = i >> 3, c8 = (i & 7) * 8;
    uint8_t* dst = tile + sw_off(r, c8);
    if (r < S) cp_async16(dst, src + (long long)r * ld + col0 + c8);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
}

ODP_DEVICE void load8f(const float* p, float (&v)[8]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// Rotate one 8-column chunk pair (columns j.. and j+32..) of a staged row in place:
//   out[j] = x[j] cos[j] - x[j+32] sin[j],  out[j+32] = x[j+32] cos[j+32] + x[j] sin[j+32]
// (bf16 in, fp32 math, bf16 out).
ODP_DEVICE void rope_pair(uint8_t* tile, int r, int j, const float (&c0)[8], const float (&s0)[8],
                          const float (&c1)[8], const float (&s1)[8]) {
  uint4* p0 = reinterpret_cast<uint4*>(tile + sw_off(r, j));
  uint4* p1 = reinterpret_cast<uint4*>(tile + sw_off(r, j + 32));
  const uint4 xv = *p0, yv = *p1;
  const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&xv);
  const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&yv);
  uint32_t a[4], b[4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const float x0 = __bfloat162float(x[e]), x1 = __bfloat162float(x[e + 1]);
    const float y0 = __bfloat162float(y[e]), y1 = __bfloat162float(y[e + 1]);
    a[e / 2] = pack_bf16(x0 * c0[e] - y0 * s0[e], x1 * c0[e + 1] - y1 * s0[e + 1]);
    b[e / 2] = pack_bf16(y0 * c1[e] + x0 * s1[e], y1 * c1[e + 1] + x1 * s1[e + 1]);
  }
  *p0 = make_uint4(a[0], a[1], a[2], a[3]);
  *p1 = make_uint4(b[0], b[1], b[2], b[3]);
}

// RoPE in place on one or two staged tiles (position = row), cos/sin loaded once per
// (row, chunk pair) with 16-byte loads and shared by both tiles.
template <int NT>
ODP_DEVICE void rope_tiles(uint8_t* t0, uint8_t* t1, int S, const float* cosT, const float* sinT) {
  for (int i = threadIdx.x; i < T * 4; i += NT) {
    const int r = i >> 2, j = (i & 3) * 8;
    if (r >= S) continue;
    float c0[8], s0[8], c1[8], s1[8];
    load8f(cosT + (long long)r * D + j, c0);
    load8f(sinT + (long long)r * D + j, s0);
    load8f(cosT + (long long)r * D + j + 32, c1);
    load8f(sinT + (long long)r * D + j + 32, s1);
    rope_pair(t0, r, j, c0, s0, c1, s1);
    if (t1) rope_pair(t1, r, j, c0, s0, c1, s1);
  }
}

// Write 16 consecutive columns [c0, c0 + 16) of row `row` (c0 % 16 == 0) into a pair of
// [128][64] tiles that together hold 128 columns.
ODP_DEVICE void put16(uint8_t* tiles, int row, int c0, const float (&v)[16]) {
  uint8_t* t = tiles + (c0 >> 6) * TILE;
  const int c = c0 & 63;
  uint4 lo = make_uint4(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]), pack_bf16(v[4], v[5]), pack_bf16(v[6], v[7]));
  uint4 hi = make_uint4(pack_bf16(v[8], v[9]), pack_bf16(v[10], v[11]), pack_bf16(v[12], v[13]),
                        pack_bf16(v[14], v[15]));
  *reinterpret_cast<uint4*>(t + sw_off(row, c)) = lo;
  *reinterpret_cast<uint4*>(t + sw_off(row, c + 8)) = hi;
}

// The same 16 columns already packed as bf16 pairs (lo = columns c0..c0+7, hi = +8..15).
ODP_DEVICE void put16_packed(uint8_t* tiles, int row, int c0, uint4 lo, uint4 hi) {
  uint8_t* t = tiles + (c0 >> 6) * TILE;
  const int c = c0 & 63;
  *reinterpret_cast<uint4*>(t + sw_off(row, c)) = lo;
  *reinterpret_cast<uint4*>(t + sw_off(row, c + 8)) = hi;
}

// Read the 64 fp32 columns [col, col + 64) of this thread's TMEM lane.
ODP_DEVICE void tmem_row64(uint32_t taddr, float (&r)[64]) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float v[16];
    tmem_ld16(taddr + c * 16, v);
#pragma unroll
    for (int e = 0; e < 16; ++e) r[c * 16 + e] = v[e];
  }
}

// Store a 64-wide fp32 row as bf16 (8 x 16-byte stores), multiplied by `mul` and, if
// asked, passed through the transpose of RoPE at position s:
//   g[i] = r[i] cos[i] + r[i+32] sin[i+32],  g[i+32] = r[i+32] cos[i+32] - r[i] sin[i]   (i < 32)
ODP_DEVICE void store_row64(__nv_bfloat16* dst, const float (&r)[64], float mul, const float* cosT,
                            const float* sinT, int s, bool rope_t) {
  uint4* out = reinterpret_cast<uint4*>(dst);
  if (!rope_t) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
      out[c] = make_uint4(pack_bf16(r[c * 8] * mul, r[c * 8 + 1] * mul), pack_bf16(r[c * 8 + 2] * mul, r[c * 8 + 3] * mul),
                          pack_bf16(r[c * 8 + 4] * mul, r[c * 8 + 5] * mul), pack_bf16(r[c * 8 + 6] * mul, r[c * 8 + 7] * mul));
    return;
  }
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float c0[8], s0[8], c1[8], s1[8], lo[8], hi[8];
    load8f(cosT + (long long)s * D + c * 8, c0);
    load8f(sinT + (long long)s * D + c * 8, s0);
    load8f(cosT + (long long)s * D + 32 + c * 8, c1);
    load8f(sinT + (long long)s * D + 32 + c * 8, s1);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float x = r[c * 8 + e] * mul, y = r[32 + c * 8 + e] * mul;
      lo[e] = x * c0[e] + y * s1[e];
      hi[e] = y * c1[e] - x * s0[e];
    }
    out[c] = make_uint4(pack_bf16(lo[0], lo[1]), pack_bf16(lo[2], lo[3]), pack_bf16(lo[4], lo[5]), pack_bf16(lo[6], lo[7]));
    out[4 + c] = make_uint4(pack_bf16(hi[0], hi[1]), pack_bf16(hi[2], hi[3]), pack_bf16(hi[4], hi[5]),
                            pack_bf16(hi[6], hi[7]));
  }
}

__global__ void __launch_bounds__(128) fwd_kernel(Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm;
  uint8_t* sK = sm + TILE;
  uint8_t* sV = sm + 2 * TILE;
  uint8_t* sP = sm;  // two tiles over Q and K, written once S = Q K^T has completed
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  const int h = blockIdx.x, gb = blockIdx.y;
  const int warp = threadIdx.x / 32, row = threadIdx.x;
  const int kvh = h / (a.nh / a.nkv);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_holder, 128);
  pdl_wait();  // global memory only from here on
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  stage_async<128>(sQ, base, a.ld, h * D, a.S);
  stage_async<128>(sK, base, a.ld, (a.nh + kvh) * D, a.S);
  stage_async<128>(sV, base, a.ld, (a.nh + a.nkv + kvh) * D, a.S);
  cp_async_wait_all();
  __syncthreads();
  rope_tiles<128>(sQ, sK, a.S, a.cosT, a.sinT);
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_holder;
  pdl_trigger();  // after this CTA's TMEM allocation
  const uint32_t trow = tm + ((uint32_t)(warp * 32) << 16);

  if (threadIdx.x == 0) {
    constexpr uint32_t idS = umma_idesc_bf16(T, T, false, false);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) umma_bf16(tm, desc_k(smem_u32(sQ), kk), desc_k(smem_u32(sK), kk), idS, kk > 0);
    umma_commit(&bar);
  }
  __syncwarp();
  // one thread waits for the MMAs (bounded); the rest sleep in the block barrier instead of
  // polling the mbarrier alongside the other CTAs of the SM
  bool ok = true;
  if (threadIdx.x == 0) ok = mbar_wait(&bar, 0, a.err, ERR_TIMEOUT_ACCUM);
  ok = __syncthreads_and(ok);
  tc_fence_after();

  const float sl2 = a.scale * kLog2e;
  const int nvalid = row < a.S ? row + 1 : 0;  // causal: keys [0, row]; padding rows see none
  // causal: chunks at or past nvalid are all masked; their TMEM loads still run (the
  // load is warp-collective) but they cost no exponentials
  float mx = -INFINITY;
#pragma unroll 1
  for (int c = 0; c < T / 16; ++c) {
    float v[16];
    tmem_ld16(trow + c * 16, v);
    if (c * 16 < nvalid) {
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c * 16 + e < nvalid) mx = fmaxf(mx, v[e] * sl2);
    }
  }
  float l = 0.f;
#pragma unroll 1
  for (int c = 0; c < T / 16; ++c) {
    float v[16];
    tmem_ld16(trow + c * 16, v);
    if (c * 16 < nvalid) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float p = (c * 16 + e < nvalid) ? ex2_fast(v[e] * sl2 - mx) : 0.f;
        v[e] = p;
        l += p;
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = 0.f;
    }
    put16(sP, row, c * 16, v);
  }
  fence_async_smem();
  tc_fence_before();
  ok = __syncthreads_and(ok);  // every thread agrees whether the second MMA is issued
  tc_fence_after();
  if (threadIdx.x == 0 && ok) {
    constexpr uint32_t idO = umma_idesc_bf16(T, D, false, true);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16(tm, desc_k(smem_u32(sP + (kk >> 2) * TILE), kk & 3), desc_mn(smem_u32(sV), kk), idO, kk > 0);
    umma_commit(&bar);
  }
  __syncwarp();
  if (ok && threadIdx.x == 0) ok = mbar_wait(&bar, 1, a.err, ERR_TIMEOUT_ACCUM);
  ok = __syncthreads_and(ok);
  tc_fence_after();
  float r[64];
  tmem_row64(trow, r);
  if (ok && row < a.S) {
    store_row64(a.o + ((long long)gb * a.S + row) * a.ldo + h * D, r, 1.f / l, nullptr, nullptr, 0, false);
    a.lse[((long long)gb * a.nh + h) * a.S + row] = (mx + log2f(l)) * kLn2;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 128);
}

template <bool LEAN>
__global__ void __launch_bounds__(256, LEAN ? 2 : 1) bwd_kernel(Args a) {
  constexpr uint32_t kCols = LEAN ? 256 : 512;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sK = sm;
  uint8_t* sV = sm + TILE;
  uint8_t* sQ = sm + 2 * TILE;
  uint8_t* sdO = sm + 3 * TILE;
  uint8_t* sP = sm + 4 * TILE;                  // 2 tiles
  uint8_t* sdS = LEAN ? sP : sm + 6 * TILE;     // 2 tiles (the lean variant reuses P's)
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  __shared__ float sDelta[T], sLse[T];
  const int kvh = blockIdx.x, gb = blockIdx.y;
  const int grp = a.nh / a.nkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int quarter = warp % 4, half = warp / 4;
  const int row = quarter * 32 + lane;  // TMEM lane / tile row this thread reads
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_holder, kCols);
  pdl_wait();  // global memory only from here on
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const __nv_bfloat16* dobase = a.dout + (long long)gb * a.S * a.ldo;
  stage_async<256>(sK, base, a.ld, (a.nh + kvh) * D, a.S);
  stage_async<256>(sV, base, a.ld, (a.nh + a.nkv + kvh) * D, a.S);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_holder;
  pdl_trigger();  // after this CTA's TMEM allocation
  const uint32_t tS = tm, tdP = tm + 128;
  const uint32_t tdV = LEAN ? tm : tm + 256, tdK = LEAN ? tm + 64 : tm + 320, tdQ = LEAN ? tm + 128 : tm + 384;
  const float sl2 = a.scale * kLog2e;
  uint32_t phase = 0;
  bool ok = true;

  for (int hi = 0; hi < grp && ok; ++hi) {
    const int h = kvh * grp + hi;
    stage_async<256>(sQ, base, a.ld, h * D, a.S);
    stage_async<256>(sdO, dobase, a.ldo, h * D, a.S);
    // this thread's O row, for delta = rowsum(dO O): loaded while the tiles stream in
    // (the lean variant keeps it packed, 32 registers instead of 64)
    uint4 opk[8];
    float orow[LEAN ? 1 : 64];
    if (threadIdx.x < T && threadIdx.x < a.S) {
      const uint4* op = reinterpret_cast<const uint4*>(a.o + ((long long)gb * a.S + threadIdx.x) * a.ldo + h * D);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 ov = op[c];
        if constexpr (LEAN) {
          opk[c] = ov;
        } else {
          const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&ov);
#pragma unroll
          for (int e = 0; e < 8; ++e) orow[c * 8 + e] = __bfloat162float(x[e]);
        }
      }
    }
    cp_async_wait_all();
    __syncthreads();
    rope_tiles<256>(sQ, hi == 0 ? sK : nullptr, a.S, a.cosT, a.sinT);
    if (threadIdx.x < T) {
      const int r = threadIdx.x;
      float dsum = 0.f, l2 = 0.f;
      if (r < a.S) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 dv = *reinterpret_cast<const uint4*>(sdO + sw_off(r, c * 8));
          const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&dv);
          const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&opk[c]);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float ov = LEAN ? __bfloat162float(x[e]) : orow[(c * 8 + e) % (LEAN ? 1 : 64)];
            dsum += ov * __bfloat162float(y[e]);
          }
        }
        l2 = a.lse[((long long)gb * a.nh + h) * a.S + r] * kLog2e;
      }
      sDelta[r] = dsum;
      sLse[r] = l2;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) {
      constexpr uint32_t idSS = umma_idesc_bf16(T, T, false, false);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_bf16(tS, desc_k(smem_u32(sQ), kk), desc_k(smem_u32(sK), kk), idSS, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tdP, desc_k(smem_u32(sdO), kk), desc_k(smem_u32(sV), kk), idSS, kk > 0);
      umma_commit(&bar);
    }
    __syncwarp();
    if (threadIdx.x == 0) ok = mbar_wait(&bar, phase, a.err, ERR_TIMEOUT_ACCUM);
    phase ^= 1;
    ok = __syncthreads_and(ok);
    tc_fence_after();
    uint4 dsk[LEAN ? 4 : 1][2];  // lean: this thread's dS (bf16 pairs) until P has been consumed
    {
      const int nvalid = row < a.S ? row + 1 : 0;
      const float delta = sDelta[row], l2 = sLse[row];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int c0 = half * 64 + c * 16;
        float s[16], dp[16];
        tmem_ld16(tS + lane_off + c0, s);
        tmem_ld16(tdP + lane_off + c0, dp);
        if (c0 < nvalid) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float p = (c0 + e < nvalid) ? ex2_fast(s[e] * sl2 - l2) : 0.f;
            s[e] = p;
            dp[e] = p * (dp[e] - delta);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) s[e] = dp[e] = 0.f;
        }
        put16(sP, row, c0, s);
        if constexpr (LEAN) {
          dsk[c][0] = make_uint4(pack_bf16(dp[0], dp[1]), pack_bf16(dp[2], dp[3]), pack_bf16(dp[4], dp[5]),
                                 pack_bf16(dp[6], dp[7]));
          dsk[c][1] = make_uint4(pack_bf16(dp[8], dp[9]), pack_bf16(dp[10], dp[11]), pack_bf16(dp[12], dp[13]),
                                 pack_bf16(dp[14], dp[15]));
        } else {
          put16(sdS, row, c0, dp);
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if constexpr (LEAN) {
      // dV = P^T dO into S's columns (every thread has read S and dP), then dS over P
      if (threadIdx.x == 0 && ok) {
        constexpr uint32_t idT = umma_idesc_bf16(T, D, true, true);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tdV, desc_mn(smem_u32(sP), kk), desc_mn(smem_u32(sdO), kk), idT, kk > 0);
        umma_commit(&bar);
      }
      __syncwarp();
      if (ok && threadIdx.x == 0) ok = mbar_wait(&bar, phase, a.err, ERR_TIMEOUT_ACCUM);
      phase ^= 1;
      ok = __syncthreads_and(ok);
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) put16_packed(sdS, row, half * 64 + c * 16, dsk[c][0], dsk[c][1]);
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
    if (threadIdx.x == 0 && ok) {
      constexpr uint32_t idT = umma_idesc_bf16(T, D, true, true);    // A^T from [query][key] tiles
      constexpr uint32_t idQ = umma_idesc_bf16(T, D, false, true);   // dS (K-major) x K (MN-major)
      if constexpr (!LEAN) {
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tdV, desc_mn(smem_u32(sP), kk), desc_mn(smem_u32(sdO), kk), idT, (hi > 0 || kk > 0));
      }
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tdK, desc_mn(smem_u32(sdS), kk), desc_mn(smem_u32(sQ), kk), idT, (hi > 0 || kk > 0));
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16(tdQ, desc_k(smem_u32(sdS + (kk >> 2) * TILE), kk & 3), desc_mn(smem_u32(sK), kk), idQ, kk > 0);
      umma_commit(&bar);
    }
    __syncwarp();
    if (ok && threadIdx.x == 0) ok = mbar_wait(&bar, phase, a.err, ERR_TIMEOUT_ACCUM);
    phase ^= 1;
    ok = __syncthreads_and(ok);
    tc_fence_after();
    if (half == 0) {
      float r[64];
      tmem_row64(tdQ + lane_off, r);
      if (ok && row < a.S)
        store_row64(a.dqkv + ((long long)gb * a.S + row) * a.ld + h * D, r, a.scale, a.cosT, a.sinT, row, true);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  {
    float r[64];
    tmem_row64((half == 0 ? tdK : tdV) + lane_off, r);
    if (ok && row < a.S) {
      __nv_bfloat16* dst = a.dqkv + ((long long)gb * a.S + row) * a.ld;
      if (half == 0) store_row64(dst + (a.nh + kvh) * D, r, a.scale, a.cosT, a.sinT, row, true);
      else store_row64(dst + (a.nh + a.nkv + kvh) * D, r, 1.f, nullptr, nullptr, 0, false);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, kCols);
}


// ============================================================================ S > 128
// Flash-style kernels for sequences longer than one tile (any S >= 1; used for S > 128).
// Same operand layout, RoPE staging, exponentials and bounded mbarrier waits as above;
// the sequence is now cut into tiles and the softmax runs online across key tiles.
//
// flash_fwd_kernel: one CTA per (128-query tile, head, sequence), 128 threads, thread t
//   owns query row t. Per 64-key tile j (causal: only keys <= the tile's last query):
//     S = Q K_j^T             -> TMEM [0, 64)     (M 128, N 64, K 64)
//     online softmax: m' = max(m, rowmax), alpha = 2^(m - m'), P = 2^(S log2e/sqrt(d) - m')
//     (bf16, over the P tile), l = alpha l + rowsum P
//     O_j = P V_j             -> TMEM [64, 128)   (M 128, N 64, K 64), acc = alpha acc + O_j
//   o = acc / l, lse = (m + log2 l) ln 2. 128 TMEM columns and 48 KB of shared memory:
//   four CTAs per SM, whose MMAs and softmax phases interleave.
// flash_bwd_dq_kernel: one CTA per (128-query tile, head, sequence), 256 threads (warp w
//   reads TMEM lanes 32 (w % 4).., columns half (w / 4) of each tile). It first computes
//   delta = rowsum(dO o) for its rows (written out for the dK/dV kernel), then per 64-key
//   tile: S = Q K_j^T, dP = dO V_j^T, dS = P (dP - delta) in shared memory,
//   dQ += dS K_j in TMEM. dQ is scaled and passed through the transpose of RoPE.
// flash_bwd_dkv_kernel: one CTA per (128-key tile, kv head, sequence), 256 threads; keys
//   are the TMEM lanes. For every query head of the kv group and every 64-query tile at
//   or after the diagonal: S^T = K Q_i^T, dP^T = V dO_i^T, P^T and dS^T = P^T (dP^T -
//   delta) written as [key][query] tiles, dV += P^T dO_i, dK += dS^T Q_i in TMEM.
//   Each CTA owns its dK / dV rows: no atomics, deterministic, and dQ comes from its own
//   kernel (the S / dP products are recomputed there rather than accumulated across
//   key tiles with atomics).
// Both backward kernels use 256 TMEM columns and 64 / 80 KB of shared memory: two CTAs
// per SM.

constexpr int KT = 64;              // keys (forward, dQ) or queries (dK / dV) per inner tile
constexpr int TILE64 = KT * 128;    // bytes of a [64][64] bf16 tile
constexpr int kFlashFwdSmem = 2 * TILE + 4 * TILE64 + 1024;  // K / V double-buffered
constexpr int kFlashDqSmem = 3 * TILE + 4 * TILE64 + 1024;  // K / V double-buffered
constexpr int kFlashDkvSmem = 4 * TILE + 4 * TILE64 + 1024;  // Q / dO double-buffered

// Stage rows [r0, r0 + nrows) of 64 columns at col0 of a [S, ld] bf16 matrix into a
// swizzled tile (tile row r = matrix row r0 + r); rows >= S are zero-filled.
template <int NT>
ODP_DEVICE void stage_rows(uint8_t* tile, const __nv_bfloat16* src, long long ld, int col0, int r0, int nrows,
                           int S) {
  for (int i = threadIdx.x; i < nrows * 8; i += NT) {
    const int r = i >> 3, c8 = (i & 7) * 8;
    uint8_t* dst = tile + sw_off(r, c8);
    if (r0 + r < S) cp_async16(dst, src + (long long)(r0 + r) * ld + col0 + c8);
    else *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
  }
}

// RoPE in place on a staged tile whose row r holds position r0 + r.
template <int NT>
ODP_DEVICE void rope_rows(uint8_t* tile, int r0, int nrows, int S, const float* cosT, const float* sinT) {
  for (int i = threadIdx.x; i < nrows * 4; i += NT) {
    const int r = i >> 2, j = (i & 3) * 8;
    const int pos = r0 + r;
    if (pos >= S) continue;
    float c0[8], s0[8], c1[8], s1[8];
    load8f(cosT + (long long)pos * D + j, c0);
    load8f(sinT + (long long)pos * D + j, s0);
    load8f(cosT + (long long)pos * D + j + 32, c1);
    load8f(sinT + (long long)pos * D + j + 32, s1);
    rope_pair(tile, r, j, c0, s0, c1, s1);
  }
}

// RoPE once per call for the flash kernels: CTA (b, head, sequence) rotates rows
// [64 b, 64 b + 64) of one q or k head with the same staging and rope_rows code the
// kernels would run on each staged tile (so the rotated values are the same bits), and
// writes them to a.qkr. Without it every query tile would rotate every key tile again
// (and every (query head, tile) pair of a kv group), reading the cos / sin tables each time.
__global__ void __launch_bounds__(128) rope_qk_kernel(Args a) {
  __shared__ __align__(1024) uint8_t tile[TILE64];
  const int r0 = blockIdx.x * KT, hd = blockIdx.y, gb = blockIdx.z;
  pdl_wait();
  pdl_trigger();
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  stage_rows<128>(tile, base, a.ld, hd * D, r0, KT, a.S);
  cp_async_wait_all();
  __syncthreads();
  rope_rows<128>(tile, r0, KT, a.S, a.cosT, a.sinT);
  __syncthreads();
  __nv_bfloat16* out = const_cast<__nv_bfloat16*>(a.qkr) + (long long)gb * a.S * a.ldr + hd * D;
  for (int i = threadIdx.x; i < KT * 8; i += 128) {
    const int r = i >> 3, c8 = (i & 7) * 8;
    if (r0 + r < a.S)
      *reinterpret_cast<uint4*>(out + (long long)(r0 + r) * a.ldr + c8) =
          *reinterpret_cast<const uint4*>(tile + sw_off(r, c8));
  }
}

// Every thread of the CTA: publish shared-memory writes to the tensor core and order the
// block around tcgen05 operations.
ODP_DEVICE void publish_smem_sync() {
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// Thread 0 waits (bounded) for the next completion of `bar`; every thread returns whether
// all waits so far succeeded.
ODP_DEVICE bool wait_mma(uint64_t* bar, uint32_t& phase, bool ok, int* err) {
  if (ok && threadIdx.x == 0) ok = mbar_wait(bar, phase, err, ERR_TIMEOUT_ACCUM);
  phase ^= 1;
  ok = __syncthreads_and(ok);
  tc_fence_after();
  return ok;
}

__global__ void __launch_bounds__(128) flash_fwd_kernel(Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm;
  uint8_t* sP = sm + TILE;
  uint8_t* sKV = sm + 2 * TILE;  // two (K, V) tile pairs: tile j + 1 streams in during tile j
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  const int nqt = (a.S + T - 1) / T;
  const int qt = nqt - 1 - (int)blockIdx.x;  // longest (latest) query tiles first
  const int h = blockIdx.y, gb = blockIdx.z;
  const int warp = threadIdx.x / 32, row = threadIdx.x;
  const int q0 = qt * T, q = q0 + row;
  const int kvh = h / (a.nh / a.nkv);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_holder, 128);
  pdl_wait();  // global memory only from here on
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const int kend = min(a.S, q0 + T);  // causal: this tile needs keys [0, kend)
  const int nkt = (kend + KT - 1) / KT;
  const bool pre = a.qkr != nullptr;  // q|k rotated already
  const __nv_bfloat16* qkb = pre ? a.qkr + (long long)gb * a.S * a.ldr : base;
  const long long qkld = pre ? a.ldr : a.ld;
  stage_rows<128>(sQ, qkb, qkld, h * D, q0, T, a.S);
  stage_rows<128>(sKV, qkb, qkld, (a.nh + kvh) * D, 0, KT, a.S);
  stage_rows<128>(sKV + TILE64, base, a.ld, (a.nh + a.nkv + kvh) * D, 0, KT, a.S);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_holder;
  pdl_trigger();  // after this CTA's TMEM allocation
  const uint32_t trow = tm + ((uint32_t)(warp * 32) << 16);
  const uint32_t tS = trow, tO = trow + 64;
  const float sl2 = a.scale * kLog2e;
  float acc[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) acc[i] = 0.f;
  float m = -INFINITY, l = 0.f;
  uint32_t phase = 0;
  bool ok = true;
  for (int j = 0; j < nkt && ok; ++j) {
    const int k0 = j * KT;
    uint8_t* sK = sKV + (j & 1) * 2 * TILE64;
    uint8_t* sV = sK + TILE64;
    cp_async_wait_all();  // tile j (issued one iteration ahead) has landed
    __syncthreads();
    if (!pre) {
      if (j == 0) rope_rows<128>(sQ, q0, T, a.S, a.cosT, a.sinT);
      rope_rows<128>(sK, k0, KT, a.S, a.cosT, a.sinT);
    }
    publish_smem_sync();
    if (threadIdx.x == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(T, KT, false, false);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_bf16(tm, desc_k(smem_u32(sQ), kk), desc_k(smem_u32(sK), kk), idS, kk > 0);
      umma_commit(&bar);
    }
    __syncwarp();
    if (j + 1 < nkt) {  // the other pair was last read by tile j - 1's MMAs, which completed
      uint8_t* nK = sKV + ((j + 1) & 1) * 2 * TILE64;
      stage_rows<128>(nK, qkb, qkld, (a.nh + kvh) * D, k0 + KT, KT, a.S);
      stage_rows<128>(nK + TILE64, base, a.ld, (a.nh + a.nkv + kvh) * D, k0 + KT, KT, a.S);
    }
    ok = wait_mma(&bar, phase, ok, a.err);
    // valid keys of this row in the tile: k0 + e <= q and k0 + e < S
    const int nvalid = q < a.S ? max(0, min(KT, min(q + 1, a.S) - k0)) : 0;
    float tmax = -INFINITY;
#pragma unroll
    for (int c = 0; c < KT / 16; ++c) {
      float v[16];
      tmem_ld16(tS + c * 16, v);
#pragma unroll
      for (int e = 0; e < 16; ++e)
        if (c * 16 + e < nvalid) tmax = fmaxf(tmax, v[e] * sl2);
    }
    const float mn = fmaxf(m, tmax);
    const float alpha = mn == -INFINITY ? 1.f : ex2_fast(m - mn);  // m = -inf -> alpha 0 (acc, l are 0 then)
    float psum = 0.f;
#pragma unroll
    for (int c = 0; c < KT / 16; ++c) {
      float v[16];
      tmem_ld16(tS + c * 16, v);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float p = (c * 16 + e < nvalid) ? ex2_fast(v[e] * sl2 - mn) : 0.f;
        v[e] = p;
        psum += p;
      }
      put16(sP, row, c * 16, v);
    }
    l = l * alpha + psum;
    m = mn;
    publish_smem_sync();
    if (threadIdx.x == 0 && ok) {
      constexpr uint32_t idO = umma_idesc_bf16(T, D, false, true);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk)
        umma_bf16(tm + 64, desc_k(smem_u32(sP), kk), desc_mn(smem_u32(sV), kk), idO, kk > 0);
      umma_commit(&bar);
    }
    __syncwarp();
    ok = wait_mma(&bar, phase, ok, a.err);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      float v[16];
      tmem_ld16(tO + c * 16, v);
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[c * 16 + e] = fmaf(acc[c * 16 + e], alpha, v[e]);
    }
    tc_fence_before();
    __syncthreads();  // every thread is done with S, O_j and the tiles before they are restaged
    tc_fence_after();
  }
  if (ok && q < a.S) {
    store_row64(a.o + ((long long)gb * a.S + q) * a.ldo + h * D, acc, 1.f / l, nullptr, nullptr, 0, false);
    a.lse[((long long)gb * a.nh + h) * a.S + q] = (m + log2f(l)) * kLn2;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 128);
}

__global__ void __launch_bounds__(256) flash_bwd_dq_kernel(Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sQ = sm;
  uint8_t* sdO = sm + TILE;
  uint8_t* sdS = sm + 2 * TILE;  // [128 queries][64 keys]
  uint8_t* sKV = sm + 3 * TILE;  // two (K, V) tile pairs: tile j + 1 streams in during tile j
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  __shared__ float sDelta[T], sLse[T];
  const int nqt = (a.S + T - 1) / T;
  const int qt = nqt - 1 - (int)blockIdx.x;
  const int h = blockIdx.y, gb = blockIdx.z;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int quarter = warp % 4, half = warp / 4;
  const int row = quarter * 32 + lane;
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  const int q0 = qt * T, q = q0 + row;
  const int kvh = h / (a.nh / a.nkv);
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_holder, 256);
  pdl_wait();  // global memory only from here on
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const __nv_bfloat16* dobase = a.dout + (long long)gb * a.S * a.ldo;
  const bool pre = a.qkr != nullptr;  // q|k rotated already
  const __nv_bfloat16* qkb = pre ? a.qkr + (long long)gb * a.S * a.ldr : base;
  const long long qkld = pre ? a.ldr : a.ld;
  stage_rows<256>(sQ, qkb, qkld, h * D, q0, T, a.S);
  stage_rows<256>(sdO, dobase, a.ldo, h * D, q0, T, a.S);
  stage_rows<256>(sKV, qkb, qkld, (a.nh + kvh) * D, 0, KT, a.S);
  stage_rows<256>(sKV + TILE64, base, a.ld, (a.nh + a.nkv + kvh) * D, 0, KT, a.S);
  // this thread's O row (threads < 128), for delta = rowsum(dO o), loaded while the tiles stream in
  uint4 opk[8];
  const int qr = q0 + (int)threadIdx.x;
  if (threadIdx.x < T && qr < a.S) {
    const uint4* op = reinterpret_cast<const uint4*>(a.o + ((long long)gb * a.S + qr) * a.ldo + h * D);
#pragma unroll
    for (int c = 0; c < 8; ++c) opk[c] = op[c];
  }
  cp_async_wait_all();
  __syncthreads();
  if (threadIdx.x < T) {
    float dsum = 0.f, l2 = 0.f;
    if (qr < a.S) {
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 dv = *reinterpret_cast<const uint4*>(sdO + sw_off(threadIdx.x, c * 8));
        const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&dv);
        const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&opk[c]);
#pragma unroll
        for (int e = 0; e < 8; ++e) dsum += __bfloat162float(x[e]) * __bfloat162float(y[e]);
      }
      const long long li = ((long long)gb * a.nh + h) * a.S + qr;
      l2 = a.lse[li] * kLog2e;
      a.delta[li] = dsum;
    }
    sDelta[threadIdx.x] = dsum;
    sLse[threadIdx.x] = l2;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_holder;
  pdl_trigger();  // after this CTA's TMEM allocation
  const uint32_t tS = tm, tdP = tm + 64, tdQ = tm + 128;
  const float sl2 = a.scale * kLog2e;
  const float delta = sDelta[row], l2 = sLse[row];
  const int kend = min(a.S, q0 + T);
  const int nkt = (kend + KT - 1) / KT;
  uint32_t phase = 0;
  bool ok = true;
  for (int j = 0; j < nkt && ok; ++j) {
    const int k0 = j * KT;
    uint8_t* sK = sKV + (j & 1) * 2 * TILE64;
    uint8_t* sV = sK + TILE64;
    cp_async_wait_all();  // tile j (issued one iteration ahead) has landed
    __syncthreads();
    if (!pre) {
      if (j == 0) rope_rows<256>(sQ, q0, T, a.S, a.cosT, a.sinT);
      rope_rows<256>(sK, k0, KT, a.S, a.cosT, a.sinT);
    }
    publish_smem_sync();
    if (threadIdx.x == 0) {
      constexpr uint32_t idS = umma_idesc_bf16(T, KT, false, false);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) umma_bf16(tS, desc_k(smem_u32(sQ), kk), desc_k(smem_u32(sK), kk), idS, kk > 0);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_bf16(tdP, desc_k(smem_u32(sdO), kk), desc_k(smem_u32(sV), kk), idS, kk > 0);
      umma_commit(&bar);
    }
    __syncwarp();
    if (j + 1 < nkt) {  // the other pair was last read by tile j - 1's MMAs, which completed
      uint8_t* nK = sKV + ((j + 1) & 1) * 2 * TILE64;
      stage_rows<256>(nK, qkb, qkld, (a.nh + kvh) * D, k0 + KT, KT, a.S);
      stage_rows<256>(nK + TILE64, base, a.ld, (a.nh + a.nkv + kvh) * D, k0 + KT, KT, a.S);
    }
    ok = wait_mma(&bar, phase, ok, a.err);
    const int nvalid = q < a.S ? max(0, min(KT, min(q + 1, a.S) - k0)) : 0;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int c0 = half * 32 + c * 16;
      float s[16], dp[16];
      tmem_ld16(tS + lane_off + c0, s);
      tmem_ld16(tdP + lane_off + c0, dp);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float p = (c0 + e < nvalid) ? ex2_fast(s[e] * sl2 - l2) : 0.f;
        dp[e] = p * (dp[e] - delta);
      }
      put16(sdS, row, c0, dp);
    }
    publish_smem_sync();
    if (threadIdx.x == 0 && ok) {
      constexpr uint32_t idQ = umma_idesc_bf16(T, D, false, true);
#pragma unroll
      for (int kk = 0; kk < KT / 16; ++kk)
        umma_bf16(tdQ, desc_k(smem_u32(sdS), kk), desc_mn(smem_u32(sK), kk), idQ, (j > 0 || kk > 0));
      umma_commit(&bar);
    }
    __syncwarp();
    ok = wait_mma(&bar, phase, ok, a.err);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  }
  if (half == 0) {
    float r[64];
    tmem_row64(tdQ + lane_off, r);
    if (ok && q < a.S)
      store_row64(a.dqkv + ((long long)gb * a.S + q) * a.ld + h * D, r, a.scale, a.cosT, a.sinT, q, true);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 256);
}

__global__ void __launch_bounds__(256) flash_bwd_dkv_kernel(Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = align1024(smem_raw);
  uint8_t* sK = sm;
  uint8_t* sV = sm + TILE;
  uint8_t* sPT = sm + 2 * TILE;   // [128 keys][64 queries]
  uint8_t* sdST = sm + 3 * TILE;  // [128 keys][64 queries]
  uint8_t* sQdO = sm + 4 * TILE;  // two (Q [64 queries][64], dO) pairs: the next streams in during this one
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_holder;
  __shared__ float sDelta2[2][KT], sLse2[2][KT];
  const int kt = blockIdx.x, kvh = blockIdx.y, gb = blockIdx.z;
  const int grp = a.nh / a.nkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int quarter = warp % 4, half = warp / 4;
  const int row = quarter * 32 + lane;
  const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
  const int k0 = kt * T, k = k0 + row;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_holder, 256);
  pdl_wait();  // global memory only from here on
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const __nv_bfloat16* dobase = a.dout + (long long)gb * a.S * a.ldo;
  const bool pre = a.qkr != nullptr;  // q|k rotated already
  const __nv_bfloat16* qkb = pre ? a.qkr + (long long)gb * a.S * a.ldr : base;
  const long long qkld = pre ? a.ldr : a.ld;
  stage_rows<256>(sK, qkb, qkld, (a.nh + kvh) * D, k0, T, a.S);
  stage_rows<256>(sV, base, a.ld, (a.nh + a.nkv + kvh) * D, k0, T, a.S);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tm = tmem_holder;
  pdl_trigger();  // after this CTA's TMEM allocation
  const uint32_t tS = tm, tdP = tm + 64, tdV = tm + 128, tdK = tm + 192;
  const float sl2 = a.scale * kLog2e;
  const int i0 = k0 / KT, nq = (a.S + KT - 1) / KT;  // query tiles at or after the diagonal
  uint32_t phase = 0;
  bool ok = true, accumulated = false;
  // iteration it = (query head hi, query tile i) in order; its Q / dO tiles, lse and delta
  // go to pair it & 1, issued one iteration ahead
  auto stage_it = [&](int hi, int i, int b) {
    const int h = kvh * grp + hi, qs = i * KT;
    uint8_t* q = sQdO + b * 2 * TILE64;
    stage_rows<256>(q, qkb, qkld, h * D, qs, KT, a.S);
    stage_rows<256>(q + TILE64, dobase, a.ldo, h * D, qs, KT, a.S);
    if (threadIdx.x < KT) {
      const int qq = qs + (int)threadIdx.x;
      const long long li = ((long long)gb * a.nh + h) * a.S + qq;
      sLse2[b][threadIdx.x] = qq < a.S ? a.lse[li] * kLog2e : 0.f;
      sDelta2[b][threadIdx.x] = qq < a.S ? a.delta[li] : 0.f;
    }
  };
  if (i0 < nq) stage_it(0, i0, 0);
  int it = 0;
  for (int hi = 0; hi < grp && ok; ++hi) {
    const int h = kvh * grp + hi;
    for (int i = i0; i < nq && ok; ++i, ++it) {
      const int qs = i * KT;
      const int b = it & 1;
      uint8_t* sQ = sQdO + b * 2 * TILE64;
      uint8_t* sdO = sQ + TILE64;
      const float* sLse = sLse2[b];
      const float* sDelta = sDelta2[b];
      cp_async_wait_all();  // this iteration's tiles (issued one iteration ahead) have landed
      __syncthreads();
      if (!pre) {
        if (hi == 0 && i == i0) rope_rows<256>(sK, k0, T, a.S, a.cosT, a.sinT);
        rope_rows<256>(sQ, qs, KT, a.S, a.cosT, a.sinT);
      }
      publish_smem_sync();
      if (threadIdx.x == 0) {
        constexpr uint32_t idS = umma_idesc_bf16(T, KT, false, false);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tS, desc_k(smem_u32(sK), kk), desc_k(smem_u32(sQ), kk), idS, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_bf16(tdP, desc_k(smem_u32(sV), kk), desc_k(smem_u32(sdO), kk), idS, kk > 0);
        umma_commit(&bar);
      }
      __syncwarp();
      {  // the other pair was last read by the previous iteration's MMAs, which completed
        const bool last_i = i + 1 >= nq;
        if (!last_i) stage_it(hi, i + 1, b ^ 1);
        else if (hi + 1 < grp) stage_it(hi + 1, i0, b ^ 1);
      }
      ok = wait_mma(&bar, phase, ok, a.err);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int c0 = half * 32 + c * 16;
        float s[16], dp[16];
        tmem_ld16(tS + lane_off + c0, s);
        tmem_ld16(tdP + lane_off + c0, dp);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const int qq = qs + c0 + e;
          const bool valid = k <= qq && qq < a.S && k < a.S;
          const float p = valid ? ex2_fast(s[e] * sl2 - sLse[c0 + e]) : 0.f;
          s[e] = p;
          dp[e] = p * (dp[e] - sDelta[c0 + e]);
        }
        put16(sPT, row, c0, s);
        put16(sdST, row, c0, dp);
      }
      publish_smem_sync();
      if (threadIdx.x == 0 && ok) {
        constexpr uint32_t idG = umma_idesc_bf16(T, D, false, true);
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk)
          umma_bf16(tdV, desc_k(smem_u32(sPT), kk), desc_mn(smem_u32(sdO), kk), idG, (accumulated || kk > 0));
#pragma unroll
        for (int kk = 0; kk < KT / 16; ++kk)
          umma_bf16(tdK, desc_k(smem_u32(sdST), kk), desc_mn(smem_u32(sQ), kk), idG, (accumulated || kk > 0));
        umma_commit(&bar);
      }
      __syncwarp();
      accumulated = true;
      ok = wait_mma(&bar, phase, ok, a.err);
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
    }
  }
  {
    float r[64];
    tmem_row64((half == 0 ? tdK : tdV) + lane_off, r);
    if (!accumulated) {
#pragma unroll
      for (int i = 0; i < 64; ++i) r[i] = 0.f;
    }
    if (ok && k < a.S) {
      __nv_bfloat16* dst = a.dqkv + ((long long)gb * a.S + k) * a.ld;
      if (half == 0) store_row64(dst + (a.nh + kvh) * D, r, a.scale, a.cosT, a.sinT, k, true);
      else store_row64(dst + (a.nh + a.nkv + kvh) * D, r, 1.f, nullptr, nullptr, 0, false);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tm, 256);
}

}  // namespace attn_tc
}  // namespace odp

static odp::attn_tc::Args tc_args(torch::Tensor qkv, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                                  torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor err) {
  TORCH_CHECK(S >= 1, "attention: S >= 1");
  TORCH_CHECK(nh % nkv == 0, "attention: heads must be a multiple of kv heads");
  TORCH_CHECK(qkv.is_contiguous() && o.is_contiguous() && lse.is_contiguous(), "attention: contiguous tensors");
  odp::attn_tc::Args a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ld = (nh + 2 * nkv) * odp::attn_tc::D;
  a.S = (int)S;
  a.nh = (int)nh;
  a.nkv = (int)nkv;
  a.cosT = cosT.data_ptr<float>();
  a.sinT = sinT.data_ptr<float>();
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.ldo = nh * odp::attn_tc::D;
  a.lse = lse.data_ptr<float>();
  a.scale = 1.0f / sqrtf((float)odp::attn_tc::D);
  a.err = err.data_ptr<int>();
  return a;
}

// qkv: [GB, S, (nh+2nkv)*64] bf16 -> o: [GB, S, nh*64] bf16, lse: [GB, nh, S] fp32
void attention_fwd_tc(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                      torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor err) {
  TORCH_CHECK(S <= odp::attn_tc::T, "attention_fwd_tc: one-tile kernel, S <= 128 (longer: attention_fwd_flash)");
  c10::cuda::CUDAGuard guard(qkv.device());
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::attn_tc::fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        odp::attn_tc::kFwdSmem));
    attr = true;
  }
  auto a = tc_args(qkv, S, nh, nkv, cosT, sinT, o, lse, err);
  dim3 grid((unsigned)nh, (unsigned)GB);
  C10_CUDA_CHECK(odp::launch_pdl((odp::attn_tc::fwd_kernel), dim3(grid), dim3(128), odp::attn_tc::kFwdSmem, at::cuda::getCurrentCUDAStream(), a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// dqkv: [GB, S, (nh+2nkv)*64] bf16, the gradient w.r.t. the pre-RoPE q|k|v
void attention_bwd_tc(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                      torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor dout, torch::Tensor dqkv,
                      torch::Tensor err) {
  TORCH_CHECK(S <= odp::attn_tc::T, "attention_bwd_tc: one-tile kernel, S <= 128 (longer: attention_bwd_flash)");
  c10::cuda::CUDAGuard guard(qkv.device());
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::attn_tc::bwd_kernel<false>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, odp::attn_tc::kBwdSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::attn_tc::bwd_kernel<true>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, odp::attn_tc::kBwdSmemLean));
    attr = true;
  }
  TORCH_CHECK(dout.is_contiguous() && dqkv.is_contiguous(), "attention: contiguous tensors");
  auto a = tc_args(qkv, S, nh, nkv, cosT, sinT, o, lse, err);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  dim3 grid((unsigned)nkv, (unsigned)GB);
  const char* env = getenv("ODP_ATTN_BWD_LEAN");
  if (nh == nkv && !(env && env[0] == '0'))
    C10_CUDA_CHECK(odp::launch_pdl((odp::attn_tc::bwd_kernel<true>), dim3(grid), dim3(256), odp::attn_tc::kBwdSmemLean, at::cuda::getCurrentCUDAStream(), a));
  else
    C10_CUDA_CHECK(odp::launch_pdl((odp::attn_tc::bwd_kernel<false>), dim3(grid), dim3(256), odp::attn_tc::kBwdSmem, at::cuda::getCurrentCUDAStream(), a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Any S >= 1 (used for S > 128): qkv [GB, S, (nh+2nkv)*64] bf16 -> o [GB, S, nh*64] bf16,
// lse [GB, nh, S] fp32.
// With `qkr` ([GB, S, (nh + nkv) * 64] bf16 scratch) q|k are rotated once into it first
// (one more launch) instead of in every staged tile.
static void rope_prepass(odp::attn_tc::Args& a, c10::optional<torch::Tensor>& qkr, int64_t GB, int64_t S,
                         int64_t nh, int64_t nkv, cudaStream_t st) {
  if (!qkr.has_value()) return;
  TORCH_CHECK(qkr->is_cuda() && qkr->scalar_type() == at::kBFloat16 && qkr->is_contiguous() &&
                  qkr->numel() >= GB * S * (nh + nkv) * odp::attn_tc::D,
              "attention: qkr must be a contiguous bf16 [GB, S, (nh + nkv) * 64] tensor");
  a.qkr = reinterpret_cast<const __nv_bfloat16*>(qkr->data_ptr());
  a.ldr = (nh + nkv) * odp::attn_tc::D;
  dim3 grid((unsigned)((S + odp::attn_tc::KT - 1) / odp::attn_tc::KT), (unsigned)(nh + nkv), (unsigned)GB);
  C10_CUDA_CHECK(odp::launch_pdl(odp::attn_tc::rope_qk_kernel, grid, dim3(128), 0, st, a));
}

void attention_fwd_flash(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                         torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor err,
                         c10::optional<torch::Tensor> qkr) {
  c10::cuda::CUDAGuard guard(qkv.device());
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::attn_tc::flash_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        odp::attn_tc::kFlashFwdSmem));
    attr = true;
  }
  TORCH_CHECK(cosT.size(0) >= S && sinT.size(0) >= S, "attention: RoPE tables shorter than S");
  auto a = tc_args(qkv, S, nh, nkv, cosT, sinT, o, lse, err);
  auto st = at::cuda::getCurrentCUDAStream();
  rope_prepass(a, qkr, GB, S, nh, nkv, st);
  const unsigned nqt = (unsigned)((S + odp::attn_tc::T - 1) / odp::attn_tc::T);
  dim3 grid(nqt, (unsigned)nh, (unsigned)GB);
  C10_CUDA_CHECK(odp::launch_pdl((odp::attn_tc::flash_fwd_kernel), dim3(grid), dim3(128), odp::attn_tc::kFlashFwdSmem, st, a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Backward for any S >= 1: dQ (and delta = rowsum(dO o) into `delta` [GB, nh, S]), then
// dK / dV, both into dqkv [GB, S, (nh+2nkv)*64] (gradients w.r.t. the pre-RoPE q|k|v).
void attention_bwd_flash(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                         torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor dout,
                         torch::Tensor delta, torch::Tensor dqkv, torch::Tensor err,
                         c10::optional<torch::Tensor> qkr) {
  c10::cuda::CUDAGuard guard(qkv.device());
  static bool attr = false;
  if (!attr) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::attn_tc::flash_bwd_dq_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, odp::attn_tc::kFlashDqSmem));
    C10_CUDA_CHECK(cudaFuncSetAttribute(odp::attn_tc::flash_bwd_dkv_kernel,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, odp::attn_tc::kFlashDkvSmem));
    attr = true;
  }
  TORCH_CHECK(dout.is_contiguous() && dqkv.is_contiguous() && delta.is_contiguous(), "attention: contiguous tensors");
  TORCH_CHECK(delta.numel() >= GB * nh * S && delta.scalar_type() == at::kFloat, "attention: delta [GB, nh, S] fp32");
  TORCH_CHECK(cosT.size(0) >= S && sinT.size(0) >= S, "attention: RoPE tables shorter than S");
  auto a = tc_args(qkv, S, nh, nkv, cosT, sinT, o, lse, err);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  a.delta = delta.data_ptr<float>();
  auto st = at::cuda::getCurrentCUDAStream();
  rope_prepass(a, qkr, GB, S, nh, nkv, st);
  const unsigned nt = (unsigned)((S + odp::attn_tc::T - 1) / odp::attn_tc::T);
  C10_CUDA_CHECK(odp::launch_pdl((odp::attn_tc::flash_bwd_dq_kernel), dim3(dim3(nt, (unsigned)nh, (unsigned)GB)), dim3(256), odp::attn_tc::kFlashDqSmem, st, a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  C10_CUDA_CHECK(odp::launch_pdl((odp::attn_tc::flash_bwd_dkv_kernel), dim3(dim3(nt, (unsigned)nkv, (unsigned)GB)), dim3(256), odp::attn_tc::kFlashDkvSmem, st, a));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
