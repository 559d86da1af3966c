// sm_100a primitives used by the attention kernels: mbarriers with bounded
// waits, TMA tile loads, tcgen05 (TMEM allocation, UMMA issue, commit,
// TMEM loads/stores) and the shared-memory / instruction descriptors that
// tcgen05.mma consumes.
//
// Every wait in this file is bounded by a %globaltimer deadline.  When a wait
// runs out it records an error code in the device error word and reports
// failure to the caller, which then skips the rest of its work so that the CTA
// reaches its teardown (TMEM dealloc) and exits; the host turns the recorded
// code into CTFA_ERR_DEVICE_TIMEOUT.  No code path traps.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ctfa {

// ---------------------------------------------------------------------------
// Device error word (code, site, block, thread).  Written at most once per
// launch sequence by the first thread that gives up waiting.
// ---------------------------------------------------------------------------
struct DeviceError {
  int code;     // 0 = none, otherwise CTFA_ERR_DEVICE_TIMEOUT
  int site;     // which wait gave up (kernel-specific id)
  int block;    // linear block index
  int thread;   // thread index in the block
};

// Defined here: the library is a single translation unit (csrc/ctfa_api.cu).
__device__ DeviceError g_device_error;

// Abort state shared by the CTA: once set, all remaining waits return false
// immediately so every warp drains to the teardown.
__device__ __forceinline__ void record_timeout(int site) {
  if (atomicCAS(&g_device_error.code, 0, 5) == 0) {
    g_device_error.site = site;
    g_device_error.block = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
    g_device_error.thread = threadIdx.x;
  }
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with the given parity.  `abort` lives in shared
// memory; once any thread of the CTA gives up, every later wait fails fast.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit_ns, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - start > limit_ns) {
        *abort = 1;
        record_timeout(site);
        return false;
      }
    }
  }
}

// The same wait executed by every lane of a converged warp; the result is
// warp-uniform (a failure on any lane fails all of them).
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort,
                                               uint64_t limit_ns, int site) {
  const bool ok = mbar_wait(bar, parity, abort, limit_ns, site);
  return __all_sync(0xffffffffu, ok);
}

// True on exactly one lane of a converged warp (elect.sync).  tcgen05.mma is
// issued by one thread; issuing it from a converged warp under this predicate
// (instead of from a lone lane of a diverged warp) keeps the MMA stream fed
// while the softmax / compute warps load the issue slots (measured: ~2.4x
// more MMA issue throughput under full ALU load on the other warps).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\telect.sync _|p, 0xffffffff;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this project: every CTA fetches its own tiles)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Plain (untiled) bulk copy of `bytes` contiguous bytes from global to shared
// memory, completing on `bar` like a tensor load.  Both addresses 16-byte
// aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Store a shared-memory tile to global memory through a tensor map (bulk
// group).  Coordinates are never negative here; rows past the tensor's extent
// are clipped by the copy engine.
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* smem_src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
// 4-D forms (the projection GEMMs address every operand as 4-D: [B, H, T, D]
// head tensors, [B, T, E] rows and [rows, cols] weights padded with 1s).
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tma_store_4d(const void* tmap, const void* smem_src, int x, int y, int z, int w) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(tmap),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z), "r"(w)
               : "memory");
}
// Element-wise add of a shared-memory tile into global memory (the copy
// engine performs the reduction; clipped like a store).
__device__ __forceinline__ void tma_reduce_add_4d(const void* tmap, const void* smem_src, int x, int y, int z,
                                                  int w) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          tmap),
      "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ void tma_store_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the committed stores have finished reading shared memory.
__device__ __forceinline__ void tma_store_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until the committed stores are complete (visible in global memory).
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Order this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA, tcgen05.mma) reads of the same bytes.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_holder)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05.mma.  D (TMEM, fp32) (+)= A * B.
//   SS: A and B are shared-memory descriptors.
//   TS: A lives in TMEM (K-major, lanes = rows), B is a shared-memory descriptor.
// kKind: 0 = kind::f16 (bf16 / fp16 inputs), 1 = kind::tf32.
// ---------------------------------------------------------------------------
template <int kKind>
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  if constexpr (kKind == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

template <int kKind>
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  if constexpr (kKind == 0) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrive on `bar` once every tcgen05 operation issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 format): start address, leading
// byte offset, stride byte offset (all >> 4), version 1 at bit 46, layout
// (swizzle) type at bits 61..63.
//   kLayoutSW128      (2): 128-byte swizzle, 16-byte granules XOR row%8.  K-major
//                          operands of every type; MN-major 16-bit operands.
//   kLayoutSW128Base32 (1): 128-byte swizzle, 32-byte granules XOR row%4.  The
//                          only MN-major layout the tensor core reads correctly
//                          for tf32 (measured: the 16-byte-granule layout gives
//                          zeros).  K rows are 128 bytes apart, SBO = 4 rows.
constexpr uint32_t kLayoutSW128 = 2;
constexpr uint32_t kLayoutSW128Base32 = 1;

__device__ __forceinline__ uint64_t make_sdesc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

__device__ __forceinline__ uint64_t make_sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  return make_sdesc(smem_addr, lbo_bytes, sbo_bytes, kLayoutSW128);
}

// K-major operand tile stored as 128-byte column blocks of `rows` rows each
// (TMA box = 128 bytes x rows, 128B swizzle).  k-step `ks` covers 32 bytes of
// the reduction dim: 16 bf16/fp16 or 8 tf32 elements.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t tile_addr, int rows, int ks) {
  return make_sdesc(tile_addr + (ks >> 2) * (rows * 128) + (ks & 3) * 32, 16, 1024, kLayoutSW128);
}

// MN-major operand tile [red_rows][N] stored as 128-byte column blocks of
// `red_rows` rows each.  k-step `ks` covers k_per rows of the reduction dim.
template <bool kTF32>
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t tile_addr, int red_rows, int ks, int k_per) {
  return make_sdesc(tile_addr + ks * k_per * 128, red_rows * 128, kTF32 ? 512 : 1024,
                    kTF32 ? kLayoutSW128Base32 : kLayoutSW128);
}

// k-step offsets (bytes from the tile start) of the two layouts above, and a
// descriptor advanced by such an offset: the start-address field holds the
// address in 16-byte units in bits 0..13, and shared-memory addresses stay
// below 256 KB, so adding offset/16 to the k-step-0 descriptor gives the
// k-step's descriptor without a carry into the other fields.  The MMA-issuing
// thread then spends one add per operand and k-step instead of rebuilding the
// descriptor.
__host__ __device__ constexpr uint32_t kmajor_offset(int rows, int ks) {
  return (uint32_t)((ks >> 2) * (rows * 128) + (ks & 3) * 32);
}
__host__ __device__ constexpr uint32_t mnmajor_offset(int ks, int k_per) { return (uint32_t)(ks * k_per * 128); }
__device__ __forceinline__ uint64_t desc_advance(uint64_t desc0, uint32_t offset_bytes) {
  return desc0 + (uint64_t)(offset_bytes >> 4);
}

// Instruction descriptor for kind::f16 / kind::tf32 with fp32 accumulation.
//   fmt: 0 = f16, 1 = bf16, 2 = tf32.  b_mn_major: B operand stored N-contiguous.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t fmt, int M, int N, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                           // D format f32
         | (fmt << 7) | (fmt << 10)          // A, B formats
         | ((a_mn_major ? 1u : 0u) << 15)    // A major
         | ((b_mn_major ? 1u : 0u) << 16)    // B major
         | ((uint32_t)(N >> 3) << 17)        // N / 8
         | ((uint32_t)(M >> 4) << 24);       // M / 16
}

// ---------------------------------------------------------------------------
// TMEM loads / stores (32 lanes x 32 consecutive columns, 32-bit cells).
// Warp w of a warpgroup may touch lanes [32*(w%4), 32*(w%4)+32).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Same load, straight into fp32 registers (no staging copy).
__device__ __forceinline__ void tmem_ld32f(uint32_t taddr, float* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]), "=f"(r[7]),
        "=f"(r[8]), "=f"(r[9]), "=f"(r[10]), "=f"(r[11]), "=f"(r[12]), "=f"(r[13]), "=f"(r[14]), "=f"(r[15]),
        "=f"(r[16]), "=f"(r[17]), "=f"(r[18]), "=f"(r[19]), "=f"(r[20]), "=f"(r[21]), "=f"(r[22]), "=f"(r[23]),
        "=f"(r[24]), "=f"(r[25]), "=f"(r[26]), "=f"(r[27]), "=f"(r[28]), "=f"(r[29]), "=f"(r[30]), "=f"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Store 32 fp32-register values (bit patterns) without a staging copy.
__device__ __forceinline__ void tmem_st32f(uint32_t taddr, const float* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(r[0]), "f"(r[1]), "f"(r[2]), "f"(r[3]), "f"(r[4]), "f"(r[5]), "f"(r[6]), "f"(r[7]), "f"(r[8]),
      "f"(r[9]), "f"(r[10]), "f"(r[11]), "f"(r[12]), "f"(r[13]), "f"(r[14]), "f"(r[15]), "f"(r[16]),
      "f"(r[17]), "f"(r[18]), "f"(r[19]), "f"(r[20]), "f"(r[21]), "f"(r[22]), "f"(r[23]), "f"(r[24]),
      "f"(r[25]), "f"(r[26]), "f"(r[27]), "f"(r[28]), "f"(r[29]), "f"(r[30]), "f"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Math helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Round fp32 to the nearest tf32 value (ties away from zero); the tensor core
// reads only the top 19 bits of each 32-bit operand.  Integer form: add half
// of the dropped 13-bit field to the magnitude bits, then clear the field (a
// carry into the exponent is the correct rounding).  Two integer-pipe
// instructions, which keeps the conversion off the pipe the exponentials use.
// Valid for finite inputs (the kernels never feed it inf or NaN).
__device__ __forceinline__ uint32_t f32_to_tf32_rna(float x) {
  return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Warpgroup register rebalancing (all four warps of a warpgroup execute the
// same instruction).  Counts are multiples of 8 in [24, 256]; the sum over the
// block must not exceed the registers it was launched with.
template <int N>
__device__ __forceinline__ void regs_increase() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_decrease() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// Programmatic dependent launch.  launch_dependents: the kernel launched next
// on the stream with programmatic serialization may start once every block of
// this grid has executed it (or exited).  wait: block until the grid this one
// depends on has completed and its memory is visible.
__device__ __forceinline__ void grid_dep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Work item `w` of an n_heads x n_ranks list whose rank 0 is the heaviest
// tile of every head, walked `chunk` heads at a time: inside a chunk the order
// is rank-major (the chunk's heaviest tiles first), so the blocks running at
// one time share a few heads' operands in L2 instead of streaming one head
// each.  chunk == n_heads is the plain rank-major order.
__device__ __forceinline__ void head_chunked_item(int w, int n_heads, int n_ranks, int chunk, int& rank, int& head) {
  const int per = chunk * n_ranks;
  const int ch = w / per, within = w - ch * per;
  const int heads = min(chunk, n_heads - ch * chunk);
  rank = within / heads;
  head = ch * chunk + within % heads;
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void red_add_f32(float* addr, float v) {
  asm volatile("red.relaxed.gpu.global.add.f32 [%0], %1;" ::"l"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void red_add_v4_f32(float* addr, float a, float b, float c, float d) {
  asm volatile("red.relaxed.gpu.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Element type -> tcgen05 MMA kind and operand format.
template <typename DT>
struct DTypeTraits;
template <>
struct DTypeTraits<float> {
  static constexpr int kKind = 1;  // kind::tf32
  static constexpr uint32_t kFmt = 2;
};
template <>
struct DTypeTraits<__nv_bfloat16> {
  static constexpr int kKind = 0;  // kind::f16
  static constexpr uint32_t kFmt = 1;
};
template <>
struct DTypeTraits<__half> {
  static constexpr int kKind = 0;
  static constexpr uint32_t kFmt = 0;
};

// TMEM allocations are powers of two, at least 32 columns.
__host__ __device__ constexpr uint32_t tmem_cols_for(int cols) {
  return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

}  // namespace ctfa
