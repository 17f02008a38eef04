// Device helpers shared by the engine's kernels: bf16 conversion, block
// reductions, mbarrier / TMA / tcgen05 inline PTX for sm_100a, and the
// bounded-wait convention every spin in this library follows.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ls {

// Error codes written to the engine's device error word. A kernel that gives up
// on a wait records its code here and returns; the host turns it into an error.
enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 1,    // consumer waited too long for a TMA stage
  kDevTimeoutEmpty = 2,   // producer waited too long for a free stage
  kDevTimeoutAcc = 3,     // epilogue waited too long for the accumulator
  kDevBadIndex = 4,       // a metadata index was out of range (access skipped)
  // 5 and 6 are unused
  kDevTimeoutPeer = 7,    // a tensor-parallel peer did not publish its partials in time
};

// Lane metadata: int32 [cap][kMetaFields], lane-major (one record per lane,
// so a role call uploads only its own lanes).
enum MetaField : int {
  kMetaToken = 0,
  kMetaPos = 1,       // sequence position of the lane's input token
  kMetaRow = 2,       // mapping row of the lane's timeline in this role/depth
  kMetaSlot = 3,      // KV slot receiving this token's K/V for this timeline
  kMetaForkRow = 4,   // parent mapping row to copy a prefix from, or -1
  kMetaForkLen = 5,   // prefix length to copy
  kMetaStateIn = 6,   // state-bank row read by this role
  kMetaStateOut = 7,  // state-bank row written by this role
  kMetaKind = 8,      // post rows: readout kind 0 q1, 1 q2, 2 final
  kMetaFirst = 9,     // post rows: the lane's q1 token, or -1
  kMetaSecond = 10,   // post rows: the lane's q2 token, or -1
  kMetaCycle = 11,    // post rows: per-request draw counter (random stream index)
  kMetaAhead = 12,    // lanes of the same timeline filled earlier in this call
  kMetaDrawRow = 13,  // post rows: index among the request's readouts of this cycle
  kMetaSeedLo = 14,   // post rows: the request's sampling seed, low / high 32 bits
  kMetaSeedHi = 15,
  kMetaReq = 16,      // post rows: the request's sampling-parameter slot
  kMetaFields = 17,
};

struct Meta {
  const int* p;
  int cap;
  __device__ __forceinline__ int get(int f, int b) const { return p[b * kMetaFields + f]; }
};

// Upper bound on mbarrier polls. try_wait itself suspends for a bounded time,
// so this caps a stuck wait at a few seconds before the kernel bails out.
constexpr uint32_t kWaitLimit = 1u << 24;

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }

// GEMM activations are stored as a bf16 (hi, lo) row pair per lane: row 2b
// holds bf16(v), row 2b+1 holds bf16(v - bf16(v)); the GEMM sums both.
__device__ __forceinline__ void store_pair(__nv_bfloat16* x, long K, int b, long i, float v) {
  const __nv_bfloat16 hi = f2bf(v);
  x[(2L * b) * K + i] = hi;
  x[(2L * b + 1) * K + i] = f2bf(v - bf2f(hi));
}

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __bfloat1622float2(p[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over the block; `red` needs blockDim.x / 32 floats. Fixed tree order, so
// the result is the same for a row whatever else runs in the batch.
__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = blockDim.x >> 5;
  float t = lane < nw ? red[lane] : 0.f;
  t = warp_sum(t);
  return t;
}

// Ticket for "last CTA to finish does the merge": call after a __syncthreads
// that follows the CTA's partial-result stores, from one thread. Release
// (cumulative over the CTA's stores ordered by the barrier) publishes them;
// acquire lets the CTA that draws the last ticket read every other CTA's
// partials (with L1-bypassing loads) after a second __syncthreads.
__device__ __forceinline__ int ticket_take(int* p) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(p) : "memory");
  return old;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) if the phase never flips.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int* err, int code) {
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  if (err) atomicExch(err, code);
  return false;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------- TMA
// 2-D tiled load of one box into shared memory, completing on `bar`.
// Coordinates: c0 = innermost (elements), c1 = rows. No multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulator.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

// 32 TMEM lanes x 8 consecutive 32-bit columns per warp.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms
// of 128 B (stride byte offset 1024), sm_100 descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset
  d |= (uint64_t)1 << 46;                 // descriptor version
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16: bf16 x bf16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
  return (1u << 4)                         // D format f32
         | (1u << 7)                       // A bf16
         | (1u << 10)                      // B bf16
         | ((uint32_t)(N >> 3) << 17)      // N / 8
         | ((uint32_t)(M >> 4) << 24);     // M / 16
}

// 16-byte asynchronous global -> shared copy; zero-fills when !valid.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(d), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Programmatic dependent launch controls (no-ops without the launch attribute).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ------------------------------------------------------------- row helpers
// The per-lane row kernels give each thread NV float4 columns and issue every
// global load before the first use, so a row costs one memory round trip per
// dependent phase rather than one per element.
__device__ __forceinline__ float4 ld_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }

__device__ __forceinline__ float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ int ld_volatile(const int* p) { return *reinterpret_cast<const volatile int*>(p); }

__device__ __forceinline__ unsigned long long gtime_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ float4 ld_bf4(const __nv_bfloat16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 a = __bfloat1622float2(h[0]), b = __bfloat1622float2(h[1]);
  return make_float4(a.x, a.y, b.x, b.y);
}

__device__ __forceinline__ float4 f4_scale(float4 v, float s, float4 w) {
  return make_float4(v.x * s * w.x, v.y * s * w.y, v.z * s * w.z, v.w * s * w.w);
}

__device__ __forceinline__ float f4_sq(float4 v) { return v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w; }

// (hi, lo) pair rows for 4 consecutive columns starting at i (i % 4 == 0).
__device__ __forceinline__ void store_pair4(__nv_bfloat16* x, long K, int b, long i, float4 v) {
  const float f[4] = {v.x, v.y, v.z, v.w};
  __nv_bfloat16 hi[4], lo[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    hi[k] = f2bf(f[k]);
    lo[k] = f2bf(f[k] - bf2f(hi[k]));
  }
  *reinterpret_cast<uint2*>(x + (2L * b) * K + i) = *reinterpret_cast<uint2*>(hi);
  *reinterpret_cast<uint2*>(x + (2L * b + 1) * K + i) = *reinterpret_cast<uint2*>(lo);
}

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11), counter = (i/4, pos, 0, 0).
__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
    const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
    c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

}  // namespace ls
