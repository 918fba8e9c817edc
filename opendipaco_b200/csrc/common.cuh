// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits,
// TMA (cp.async.bulk.tensor) loads, tcgen05 (TMEM alloc / MMA / commit / ld),
// bf16 conversions and warp reductions.
//
// Every wait on an mbarrier or on a flag another agent writes is bounded by a
// %globaltimer deadline. A wait that runs out records a code in the kernel's
// error word (a device int the host reads after the launch) and returns false, so
// the kernel can drain its own in-flight copies, free TMEM and return instead of
// hanging the GPU.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#include <utility>

#define ODP_DEVICE __device__ __forceinline__

namespace odp {

// ---------------------------------------------------------------- error word
enum ErrCode : int {
  ERR_NONE = 0,
  ERR_TIMEOUT_FULL = 1,      // consumer waited too long for a TMA stage
  ERR_TIMEOUT_EMPTY = 2,     // producer waited too long for a free stage
  ERR_TIMEOUT_ACCUM = 3,     // epilogue waited too long for an accumulator
  ERR_TIMEOUT_TMEM_FREE = 4, // MMA warp waited too long for the epilogue
  ERR_TIMEOUT_PEER = 5,      // a cross-GPU flag never arrived
  ERR_BAD_ARGS = 6,
};

// Default bound of any single wait: 2 s of wall time (a healthy wait is < 1 ms).
constexpr unsigned long long kWaitBoundNs = 2000000000ull;

// Bound of the waits on flags that OTHER GPUs write (cross-GPU barriers of the outer step
// and of intra-path data parallelism). Host state of this library (one value per process),
// passed to every such kernel as a launch argument, so a launch captured in a CUDA graph
// keeps the bound it was captured with. Set through `set_peer_wait_ns`.
inline unsigned long long& peer_wait_bound_ns() {
  static unsigned long long v = kWaitBoundNs;
  return v;
}

ODP_DEVICE unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

ODP_DEVICE void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------- smem addr
ODP_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
ODP_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

ODP_DEVICE void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

ODP_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar))
               : "memory");
}

ODP_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

ODP_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.
ODP_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code,
                          unsigned long long bound_ns = kWaitBoundNs) {
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > bound_ns) {
      record_error(err, code);
      return false;
    }
  }
}

// The same wait with cluster-scope acquire: for a phase completed by arrivals of the
// peer CTA of a pair (its shared-memory writes, released at cluster scope, are then
// visible to what this thread issues next, tensor-core reads included).
ODP_DEVICE bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
ODP_DEVICE bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code,
                                  unsigned long long bound_ns = kWaitBoundNs) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  unsigned long long t0 = globaltimer();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - t0 > bound_ns) {
      record_error(err, code);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
ODP_DEVICE void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 3-D tiled load (x innermost). No multicast: loads always come from this GPU's memory.
ODP_DEVICE void tma_load_3d(const CUtensorMap* m, uint64_t* bar, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 3-D tiled store shared -> global (bulk-group completion). The destination is this
// GPU's memory; x (innermost coordinate) must be a multiple of 16 bytes.
ODP_DEVICE void tma_store_3d(const CUtensorMap* m, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
ODP_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until every committed bulk store has finished READING shared memory.
ODP_DEVICE void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until every committed bulk store has completed.
ODP_DEVICE void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Make this thread's generic-proxy shared-memory writes visible to the async proxy.
ODP_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05
// UMMA shared-memory descriptor (sm100): start>>4 [0,14), LBO>>4 [16,30),
// SBO>>4 [32,46), version=1 [46,48), base offset [49,52), layout [61,64).
ODP_DEVICE uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 0x7) << 61;
  return d;
}
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW64 = 4;

// Instruction descriptor, kind::f16, bf16 x bf16 -> f32.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4)                       // D = f32
         | (1u << 7)                     // A = bf16
         | (1u << 10)                    // B = bf16
         | ((a_mn ? 1u : 0u) << 15)      // A major
         | ((b_mn ? 1u : 0u) << 16)      // B major
         | ((uint32_t)(N >> 3) << 17)    // N >> 3
         | ((uint32_t)(M >> 4) << 24);   // M >> 4
}

ODP_DEVICE void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

ODP_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

ODP_DEVICE void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05.mma of this thread completes.
ODP_DEVICE void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

ODP_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
ODP_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
ODP_DEVICE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Issue a 16-column TMEM load without waiting (pair with tmem_wait_tie*).
ODP_DEVICE void tmem_ld16_nw(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

#define ODP_TIE16(r)                                                                                        \
  "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), \
      "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])

// Wait for all outstanding TMEM loads; the registers are tied so no use of them can
// be scheduled before the wait.
ODP_DEVICE void tmem_wait_tie32(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : ODP_TIE16(r) : : "memory");
  asm volatile("" : ODP_TIE16((r + 16)) : : "memory");
}
ODP_DEVICE void reg_tie32(uint32_t* r) {
  asm volatile("" : ODP_TIE16(r) : : "memory");
  asm volatile("" : ODP_TIE16((r + 16)) : : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
ODP_DEVICE uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of both CTAs of the cluster (unconditional call sites only).
ODP_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of `p` (a shared variable of this CTA) in CTA `rank` of the cluster.
ODP_DEVICE uint32_t mapa_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
ODP_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Pair TMA load (no multicast): this CTA's tile lands in its own shared memory, the byte
// count completes on the mbarrier at `bar_cluster` (the leader CTA's barrier).
ODP_DEVICE void tma_load_3d_pair(const CUtensorMap* m, uint32_t bar_cluster, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
ODP_DEVICE void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
ODP_DEVICE void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// M = 256 MMA over the CTA pair (issued by the leader; A rows and B rows are split
// between the two CTAs' shared memory at the same offsets; D rows split across TMEMs).
ODP_DEVICE void umma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// Arrive on the mbarrier at this offset in both CTAs of the pair once the leader's
// previously issued MMAs complete (multicast of the commit, not of any load).
ODP_DEVICE void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((unsigned short)0x3)
      : "memory");
}

// ---------------------------------------------------------------- misc
ODP_DEVICE float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }

// ---------------------------------------------------------------- cross-entropy gradient
// dlogits of one row with natural log-sum-exp l and batch scale sc (1 / valid labels):
//   d = exp(x - l) * sc = 2^(x log2e - ob),  ob = l log2e - log2(sc),
// the label's column minus sc. The CE kernels and the LM-head gradient GEMMs (which form
// dlogits from the logits while staging their A operand) share these two functions, so
// both produce the same bits.
constexpr float kCeLog2e = 1.4426950408889634f;
ODP_DEVICE float ce_ob(float l, float sc) { return __fmaf_rn(l, kCeLog2e, -log2f(sc)); }
ODP_DEVICE float ce_exp(float x, float ob) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(__fmaf_rn(x, kCeLog2e, -ob)));
  return y;
}

ODP_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

ODP_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

ODP_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

ODP_DEVICE bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n .reg .b32 r;\n .reg .pred p;\n elect.sync r|p, 0xffffffff;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- programmatic dependent launch
// The kernels of an inner step run back to back in one stream (and one CUDA graph). With
// programmatic dependent launch a kernel's CTAs may start while the previous kernel's last
// CTAs still run: they do their prologue (barrier init, TMEM allocation, descriptor
// prefetch) and then block in pdl_wait() until the previous grid has completed and its
// writes are visible. Rules every kernel launched with launch_pdl() follows:
//   * no global-memory access (read or write) before pdl_wait();
//   * pdl_trigger() (which lets the NEXT kernel begin launching) only after this CTA's own
//     TMEM allocation, so a dependent CTA can never hold TMEM that a CTA of this grid
//     still needs.
// Without a preceding programmatic dependency pdl_wait() returns at once.
ODP_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
ODP_DEVICE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Whether launch_pdl() sets the programmatic-serialization attribute (ODP_PDL=0 turns it
// off for comparison runs); read once per process.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("ODP_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

// Launch `kern` in `st` allowing it to overlap the previous kernel's tail (see above).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

}  // namespace odp
