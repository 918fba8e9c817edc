// Causal self-attention for head_dim 64 with GQA, reading q/k/v straight out of the
// fused QKV projection output [G*B, S, (nh + 2*nkv) * 64] (bf16).
//
// RoPE (rotate-half, fp32 cos/sin tables) is applied while Q and K tiles are staged
// into shared memory (bf16 in -> fp32 rotate -> bf16, the same rounding points as a
// bf16-autocast Llama layer), and its transpose is applied to dQ/dK before they are
// stored, so the projection GEMMs never see a separate RoPE pass.
//
// Forward: one CTA per (64-query block, head, sequence); 4 warps x 16 query rows;
// online softmax in base 2; writes O (bf16) and the row log-sum-exp (fp32).
// Backward is split in two kernels so no float atomics are needed:
//   dkdv: one CTA per (64-key block, kv head, sequence), loops over the kv group's
//         query heads and the query blocks at or after the key block;
//   dq:   one CTA per (64-query block, head, sequence), loops over key blocks.
// Both recompute P from the saved log-sum-exp. Tensor-core work uses
// mma.sync.m16n8k16 (bf16 in, fp32 accumulate) with ldmatrix from XOR-swizzled
// shared memory.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "common.cuh"

namespace odp {
namespace attn {

constexpr int D = 64;
constexpr int BLK = 64;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// [64 rows][64 bf16] tile, 16-byte chunks XOR-swizzled by (row & 7).
ODP_DEVICE uint32_t tile_off(int row, int col) {
  const int chunk = (col >> 3) ^ (row & 7);
  return (uint32_t)(row * 128 + chunk * 16 + (col & 7) * 2);
}

ODP_DEVICE void ldm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
ODP_DEVICE void ldm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

ODP_DEVICE void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragments (16 rows x 64 k) of rows [r0, r0+16) of a swizzled tile.
ODP_DEVICE void load_a_frags(const uint8_t* tile, int r0, uint32_t (&f)[4][4]) {
  const int lane = threadIdx.x % 32;
  const uint32_t base = smem_u32(tile);
#pragma unroll
  for (int kc = 0; kc < 4; ++kc) {
    const int row = r0 + (lane % 16), col = kc * 16 + (lane / 16) * 8;
    ldm_x4(base + tile_off(row, col), f[kc][0], f[kc][1], f[kc][2], f[kc][3]);
  }
}

// B fragments for two n-tiles (n rows [n0, n0+16)) at k chunk kc from a [n][k] tile.
ODP_DEVICE void load_b_nk(const uint8_t* tile, int n0, int kc, uint32_t& b0, uint32_t& b1, uint32_t& b2,
                          uint32_t& b3) {
  const int lane = threadIdx.x % 32;
  const int n = n0 + (lane / 16) * 8 + (lane % 8), k = kc * 16 + ((lane / 8) % 2) * 8;
  ldm_x4(smem_u32(tile) + tile_off(n, k), b0, b1, b2, b3);
}

// B fragments for two n-tiles (n cols [n0, n0+16)) at k chunk kc from a [k][n] tile.
ODP_DEVICE void load_b_kn(const uint8_t* tile, int n0, int kc, uint32_t& b0, uint32_t& b1, uint32_t& b2,
                          uint32_t& b3) {
  const int lane = threadIdx.x % 32;
  const int k = kc * 16 + (lane % 8) + ((lane / 8) % 2) * 8, n = n0 + (lane / 16) * 8;
  ldm_x4_t(smem_u32(tile) + tile_off(k, n), b0, b1, b2, b3);
}

// Stage 64 rows x 64 cols of head `col0` from a [S, ld] bf16 matrix into a swizzled
// tile, optionally rotating (RoPE) with the cos/sin tables at positions row0 + r.
ODP_DEVICE void stage_tile(uint8_t* tile, const __nv_bfloat16* src, long long ld, int row0, int col0, int S,
                           const float* cosT, const float* sinT, bool rope) {
  // 128 threads; each handles 8 consecutive columns of one row per iteration (4 per row pair)
  for (int i = threadIdx.x; i < BLK * 8; i += blockDim.x) {
    const int r = i / 8, c8 = (i % 8) * 8;
    const int s = row0 + r;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (s < S) {
      const __nv_bfloat16* rowp = src + (long long)s * ld + col0;
      val = *reinterpret_cast<const uint4*>(rowp + c8);
      if (rope) {
        const int pc = c8 < 32 ? c8 + 32 : c8 - 32;  // partner columns (rotate half)
        uint4 pv = *reinterpret_cast<const uint4*>(rowp + pc);
        const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&val);
        const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&pv);
        const float* cs = cosT + (long long)s * D + c8;
        const float* sn = sinT + (long long)s * D + c8;
        const float sign = c8 < 32 ? -1.f : 1.f;
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          float v0 = __bfloat162float(x[e]) * cs[e] + sign * __bfloat162float(y[e]) * sn[e];
          float v1 = __bfloat162float(x[e + 1]) * cs[e + 1] + sign * __bfloat162float(y[e + 1]) * sn[e + 1];
          o[e / 2] = pack_bf16(v0, v1);
        }
        val = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
    *reinterpret_cast<uint4*>(tile + tile_off(r, c8)) = val;
  }
}

// Store a warp's 16 x 64 fp32 accumulator (rows r0.., 8 n-tiles) as bf16, optionally
// applying the transpose of RoPE (for dQ / dK) at positions pos0 + row.
ODP_DEVICE void store_rows(const float (&acc)[8][4], __nv_bfloat16* dst, long long ld, int pos0, int r0, int S,
                           float mul, const float* cosT, const float* sinT, bool rope_t) {
  const int lane = threadIdx.x % 32, g = lane / 4, c = (lane % 4) * 2;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int row = r0 + g + half * 8;
    const int s = pos0 + row;
    if (s >= S) continue;
    __nv_bfloat16* rp = dst + (long long)s * ld;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      float v[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = nt * 8 + c + e;
        float x = acc[nt][half * 2 + e] * mul;
        if (rope_t) {
          // dq[i] = dr[i] cos[i] + dr[i+32] sin[i+32]   (i < 32)
          // dq[i] = dr[i] cos[i] - dr[i-32] sin[i-32]   (i >= 32)
          const int pn = nt < 4 ? nt + 4 : nt - 4;
          const int pcol = pn * 8 + c + e;
          const float xp = acc[pn][half * 2 + e] * mul;
          const float cs = cosT[(long long)s * D + col];
          const float sp = sinT[(long long)s * D + pcol];
          x = nt < 4 ? x * cs + xp * sp : x * cs - xp * sp;
        }
        v[e] = x;
      }
      *reinterpret_cast<uint32_t*>(rp + nt * 8 + c) = pack_bf16(v[0], v[1]);
    }
  }
}

// Convert a 16 x 64 accumulator (8 n-tiles) into 4 A fragments (k chunks of 16).
ODP_DEVICE void acc_to_a(const float (&s)[8][4], uint32_t (&a)[4][4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    a[j][0] = pack_bf16(s[2 * j][0], s[2 * j][1]);
    a[j][1] = pack_bf16(s[2 * j][2], s[2 * j][3]);
    a[j][2] = pack_bf16(s[2 * j + 1][0], s[2 * j + 1][1]);
    a[j][3] = pack_bf16(s[2 * j + 1][2], s[2 * j + 1][3]);
  }
}

struct Args {
  const __nv_bfloat16* qkv;
  long long ld;  // row stride of qkv (elements) = (nh + 2 nkv) * 64
  int S, nh, nkv;
  const float* cosT;
  const float* sinT;
  __nv_bfloat16* o;
  long long ldo;  // nh * 64
  float* lse;     // [GB][nh][S]
  const __nv_bfloat16* dout;
  float* delta;   // [GB][nh][S]
  __nv_bfloat16* dqkv;
  float scale;
};

__global__ void __launch_bounds__(128) fwd_kernel(Args a) {
  __shared__ __align__(128) uint8_t sQ[BLK * 128];
  __shared__ __align__(128) uint8_t sK[BLK * 128];
  __shared__ __align__(128) uint8_t sV[BLK * 128];
  const int qb = blockIdx.x, h = blockIdx.y, gb = blockIdx.z;
  const int kvh = h / (a.nh / a.nkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, c = (lane % 4) * 2;
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const int kcol = (a.nh + kvh) * D, vcol = (a.nh + a.nkv + kvh) * D;
  stage_tile(sQ, base, a.ld, qb * BLK, h * D, a.S, a.cosT, a.sinT, true);
  __syncthreads();
  uint32_t qf[4][4];
  load_a_frags(sQ, warp * 16, qf);
  const float sl2 = a.scale * kLog2e;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float oacc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
  const int q_row0 = qb * BLK + warp * 16 + g;
  for (int kb = 0; kb <= qb; ++kb) {
    __syncthreads();
    stage_tile(sK, base, a.ld, kb * BLK, kcol, a.S, a.cosT, a.sinT, true);
    stage_tile(sV, base, a.ld, kb * BLK, vcol, a.S, nullptr, nullptr, false);
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_nk(sK, np * 16, kc, b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kc], b0, b1);
        mma16816(s[2 * np + 1], qf[kc], b2, b3);
      }
    }
    float mx[2] = {m[0], m[1]};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * BLK + nt * 8 + c + (e & 1);
        const int qrow = q_row0 + (e >> 1) * 8;
        float x = s[nt][e] * sl2;
        if (key > qrow || key >= a.S) x = -INFINITY;
        s[nt][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 1));
      mx[hh] = fmaxf(mx[hh], __shfl_xor_sync(0xffffffffu, mx[hh], 2));
    }
    float corr[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) corr[hh] = exp2f(m[hh] - mx[hh]);
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[nt][e] - mx[e >> 1]);
        s[nt][e] = p;
        rs[e >> 1] += p;
      }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      l[hh] = l[hh] * corr[hh] + rs[hh];
      m[hh] = mx[hh];
    }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      oacc[nt][0] *= corr[0];
      oacc[nt][1] *= corr[0];
      oacc[nt][2] *= corr[1];
      oacc[nt][3] *= corr[1];
    }
    uint32_t pa[4][4];
    acc_to_a(s, pa);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_kn(sV, np * 16, kc, b0, b1, b2, b3);
        mma16816(oacc[2 * np], pa[kc], b0, b1);
        mma16816(oacc[2 * np + 1], pa[kc], b2, b3);
      }
    }
  }
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    l[hh] += __shfl_xor_sync(0xffffffffu, l[hh], 1);
    l[hh] += __shfl_xor_sync(0xffffffffu, l[hh], 2);
  }
  float inv[2] = {1.f / l[0], 1.f / l[1]};
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    oacc[nt][0] *= inv[0];
    oacc[nt][1] *= inv[0];
    oacc[nt][2] *= inv[1];
    oacc[nt][3] *= inv[1];
  }
  __nv_bfloat16* obase = a.o + (long long)gb * a.S * a.ldo + h * D;
  store_rows(oacc, obase, a.ldo, qb * BLK, warp * 16, a.S, 1.f, nullptr, nullptr, false);
  if ((lane % 4) == 0) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int s = q_row0 + hh * 8;
      if (s < a.S) a.lse[((long long)gb * a.nh + h) * a.S + s] = m[hh] * kLn2 + logf(l[hh]);
    }
  }
}

// delta[gb][h][s] = sum_d dO * O
__global__ void delta_kernel(Args a, int total_rows) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) / 32, lane = threadIdx.x % 32;
  if (w >= total_rows) return;
  const int s = w % a.S, h = (w / a.S) % a.nh, gb = w / (a.S * a.nh);
  const long long off = ((long long)gb * a.S + s) * a.ldo + h * D;
  const __nv_bfloat162 o = reinterpret_cast<const __nv_bfloat162*>(a.o + off)[lane];
  const __nv_bfloat162 d = reinterpret_cast<const __nv_bfloat162*>(a.dout + off)[lane];
  float v = __bfloat162float(o.x) * __bfloat162float(d.x) + __bfloat162float(o.y) * __bfloat162float(d.y);
  v = warp_sum(v);
  if (lane == 0) a.delta[((long long)gb * a.nh + h) * a.S + s] = v;
}

__global__ void __launch_bounds__(128) dkdv_kernel(Args a) {
  __shared__ __align__(128) uint8_t sK[BLK * 128];
  __shared__ __align__(128) uint8_t sV[BLK * 128];
  __shared__ __align__(128) uint8_t sQ[BLK * 128];
  __shared__ __align__(128) uint8_t sO[BLK * 128];  // dO tile
  __shared__ float sL[BLK], sD[BLK];
  const int kb = blockIdx.x, kvh = blockIdx.y, gb = blockIdx.z;
  const int grp = a.nh / a.nkv;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, c = (lane % 4) * 2;
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const __nv_bfloat16* dobase = a.dout + (long long)gb * a.S * a.ldo;
  const int kcol = (a.nh + kvh) * D, vcol = (a.nh + a.nkv + kvh) * D;
  stage_tile(sK, base, a.ld, kb * BLK, kcol, a.S, a.cosT, a.sinT, true);
  stage_tile(sV, base, a.ld, kb * BLK, vcol, a.S, nullptr, nullptr, false);
  __syncthreads();
  uint32_t kf[4][4], vf[4][4];
  load_a_frags(sK, warp * 16, kf);
  load_a_frags(sV, warp * 16, vf);
  const float sl2 = a.scale * kLog2e;
  float dk[8][4], dv[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;
  const int key0 = kb * BLK + warp * 16 + g;
  const int nqb = (a.S + BLK - 1) / BLK;
  for (int hi = 0; hi < grp; ++hi) {
    const int h = kvh * grp + hi;
    for (int qb = kb; qb < nqb; ++qb) {
      __syncthreads();
      stage_tile(sQ, base, a.ld, qb * BLK, h * D, a.S, a.cosT, a.sinT, true);
      stage_tile(sO, dobase, a.ldo, qb * BLK, h * D, a.S, nullptr, nullptr, false);
      for (int i = threadIdx.x; i < BLK; i += blockDim.x) {
        const int s = qb * BLK + i;
        const long long li = ((long long)gb * a.nh + h) * a.S + s;
        sL[i] = s < a.S ? a.lse[li] * kLog2e : INFINITY;
        sD[i] = s < a.S ? a.delta[li] : 0.f;
      }
      __syncthreads();
      // S^T = K Q^T  (16 keys x 64 queries)
      float st[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) st[i][0] = st[i][1] = st[i][2] = st[i][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc)
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          load_b_nk(sQ, np * 16, kc, b0, b1, b2, b3);
          mma16816(st[2 * np], kf[kc], b0, b1);
          mma16816(st[2 * np + 1], kf[kc], b2, b3);
        }
      // P^T
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ql = nt * 8 + c + (e & 1);
          const int q = qb * BLK + ql;
          const int key = key0 + (e >> 1) * 8;
          float p = exp2f(st[nt][e] * sl2 - sL[ql]);
          if (key > q || q >= a.S || key >= a.S) p = 0.f;
          st[nt][e] = p;
        }
      uint32_t pa[4][4];
      acc_to_a(st, pa);
      // dV += P^T dO
#pragma unroll
      for (int kc = 0; kc < 4; ++kc)
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          load_b_kn(sO, np * 16, kc, b0, b1, b2, b3);
          mma16816(dv[2 * np], pa[kc], b0, b1);
          mma16816(dv[2 * np + 1], pa[kc], b2, b3);
        }
      // dP^T = V dO^T
      float dpt[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) dpt[i][0] = dpt[i][1] = dpt[i][2] = dpt[i][3] = 0.f;
#pragma unroll
      for (int kc = 0; kc < 4; ++kc)
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          load_b_nk(sO, np * 16, kc, b0, b1, b2, b3);
          mma16816(dpt[2 * np], vf[kc], b0, b1);
          mma16816(dpt[2 * np + 1], vf[kc], b2, b3);
        }
      // dS^T = P^T (dP^T - delta)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int ql = nt * 8 + c + (e & 1);
          dpt[nt][e] = st[nt][e] * (dpt[nt][e] - sD[ql]);
        }
      uint32_t da[4][4];
      acc_to_a(dpt, da);
      // dK += dS^T Q
#pragma unroll
      for (int kc = 0; kc < 4; ++kc)
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          uint32_t b0, b1, b2, b3;
          load_b_kn(sQ, np * 16, kc, b0, b1, b2, b3);
          mma16816(dk[2 * np], da[kc], b0, b1);
          mma16816(dk[2 * np + 1], da[kc], b2, b3);
        }
    }
  }
  __nv_bfloat16* dbase = a.dqkv + (long long)gb * a.S * a.ld;
  store_rows(dk, dbase + kcol, a.ld, kb * BLK, warp * 16, a.S, a.scale, a.cosT, a.sinT, true);
  store_rows(dv, dbase + vcol, a.ld, kb * BLK, warp * 16, a.S, 1.f, nullptr, nullptr, false);
}

__global__ void __launch_bounds__(128) dq_kernel(Args a) {
  __shared__ __align__(128) uint8_t sQ[BLK * 128];
  __shared__ __align__(128) uint8_t sO[BLK * 128];
  __shared__ __align__(128) uint8_t sK[BLK * 128];
  __shared__ __align__(128) uint8_t sV[BLK * 128];
  const int qb = blockIdx.x, h = blockIdx.y, gb = blockIdx.z;
  const int kvh = h / (a.nh / a.nkv);
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, g = lane / 4, c = (lane % 4) * 2;
  const __nv_bfloat16* base = a.qkv + (long long)gb * a.S * a.ld;
  const __nv_bfloat16* dobase = a.dout + (long long)gb * a.S * a.ldo;
  const int kcol = (a.nh + kvh) * D, vcol = (a.nh + a.nkv + kvh) * D;
  stage_tile(sQ, base, a.ld, qb * BLK, h * D, a.S, a.cosT, a.sinT, true);
  stage_tile(sO, dobase, a.ldo, qb * BLK, h * D, a.S, nullptr, nullptr, false);
  __syncthreads();
  uint32_t qf[4][4], of[4][4];
  load_a_frags(sQ, warp * 16, qf);
  load_a_frags(sO, warp * 16, of);
  const int q_row0 = qb * BLK + warp * 16 + g;
  float lse2[2], dl[2];
#pragma unroll
  for (int hh = 0; hh < 2; ++hh) {
    const int s = q_row0 + hh * 8;
    const long long li = ((long long)gb * a.nh + h) * a.S + s;
    lse2[hh] = s < a.S ? a.lse[li] * kLog2e : INFINITY;
    dl[hh] = s < a.S ? a.delta[li] : 0.f;
  }
  const float sl2 = a.scale * kLog2e;
  float dq[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  for (int kb = 0; kb <= qb; ++kb) {
    __syncthreads();
    stage_tile(sK, base, a.ld, kb * BLK, kcol, a.S, a.cosT, a.sinT, true);
    stage_tile(sV, base, a.ld, kb * BLK, vcol, a.S, nullptr, nullptr, false);
    __syncthreads();
    float s[8][4], dp[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_nk(sK, np * 16, kc, b0, b1, b2, b3);
        mma16816(s[2 * np], qf[kc], b0, b1);
        mma16816(s[2 * np + 1], qf[kc], b2, b3);
        load_b_nk(sV, np * 16, kc, b0, b1, b2, b3);
        mma16816(dp[2 * np], of[kc], b0, b1);
        mma16816(dp[2 * np + 1], of[kc], b2, b3);
      }
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = kb * BLK + nt * 8 + c + (e & 1);
        const int hh = e >> 1;
        const int q = q_row0 + hh * 8;
        float p = exp2f(s[nt][e] * sl2 - lse2[hh]);
        if (key > q || key >= a.S || q >= a.S) p = 0.f;
        s[nt][e] = p * (dp[nt][e] - dl[hh]);
      }
    uint32_t da[4][4];
    acc_to_a(s, da);
#pragma unroll
    for (int kc = 0; kc < 4; ++kc)
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t b0, b1, b2, b3;
        load_b_kn(sK, np * 16, kc, b0, b1, b2, b3);
        mma16816(dq[2 * np], da[kc], b0, b1);
        mma16816(dq[2 * np + 1], da[kc], b2, b3);
      }
  }
  __nv_bfloat16* dbase = a.dqkv + (long long)gb * a.S * a.ld;
  store_rows(dq, dbase + h * D, a.ld, qb * BLK, warp * 16, a.S, a.scale, a.cosT, a.sinT, true);
}

}  // namespace attn
}  // namespace odp

static odp::attn::Args make_args(torch::Tensor qkv, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                                 torch::Tensor sinT, torch::Tensor o, torch::Tensor lse) {
  TORCH_CHECK(nh % nkv == 0, "attention: heads must be a multiple of kv heads");
  odp::attn::Args a{};
  a.qkv = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  a.ld = (nh + 2 * nkv) * odp::attn::D;
  a.S = (int)S;
  a.nh = (int)nh;
  a.nkv = (int)nkv;
  a.cosT = cosT.data_ptr<float>();
  a.sinT = sinT.data_ptr<float>();
  a.o = reinterpret_cast<__nv_bfloat16*>(o.data_ptr());
  a.ldo = nh * odp::attn::D;
  a.lse = lse.data_ptr<float>();
  a.scale = 1.0f / sqrtf((float)odp::attn::D);
  return a;
}

// qkv: [GB, S, (nh+2nkv)*64] bf16 -> o: [GB, S, nh*64] bf16, lse: [GB, nh, S] fp32
void attention_fwd(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                   torch::Tensor sinT, torch::Tensor o, torch::Tensor lse) {
  c10::cuda::CUDAGuard guard(qkv.device());
  auto a = make_args(qkv, S, nh, nkv, cosT, sinT, o, lse);
  dim3 grid((unsigned)((S + 63) / 64), (unsigned)nh, (unsigned)GB);
  odp::attn::fwd_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void attention_bwd(torch::Tensor qkv, int64_t GB, int64_t S, int64_t nh, int64_t nkv, torch::Tensor cosT,
                   torch::Tensor sinT, torch::Tensor o, torch::Tensor lse, torch::Tensor dout, torch::Tensor delta,
                   torch::Tensor dqkv) {
  c10::cuda::CUDAGuard guard(qkv.device());
  auto st = at::cuda::getCurrentCUDAStream();
  auto a = make_args(qkv, S, nh, nkv, cosT, sinT, o, lse);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  a.delta = delta.data_ptr<float>();
  a.dqkv = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  const int rows = (int)(GB * nh * S);
  odp::attn::delta_kernel<<<(rows * 32 + 255) / 256, 256, 0, st>>>(a, rows);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  dim3 g1((unsigned)((S + 63) / 64), (unsigned)nkv, (unsigned)GB);
  odp::attn::dkdv_kernel<<<g1, 128, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  dim3 g2((unsigned)((S + 63) / 64), (unsigned)nh, (unsigned)GB);
  odp::attn::dq_kernel<<<g2, 128, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}
