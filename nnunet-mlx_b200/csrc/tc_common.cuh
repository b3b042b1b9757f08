// Shared sm_100a helpers of the tensor-core kernels: mbarriers with bounded
// waits, bulk copies, TMEM loads/stores, UMMA descriptors and MMA issue.
// Included by tc_conv.cu (one translation unit for all tensor-core kernels),
// which defines nnb::g_device_status / g_device_status_where first.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace nnb {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;                            // input channels per K-step (128 bytes of fp32)
constexpr int kTmemCols = 512;
constexpr int kMaxSmem = 227 * 1024;
constexpr int kMaxKsteps = 1024;                  // K-step table capacity (taps x 32-channel chunks)
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// try_wait with a suspend-time hint: a waiting thread sleeps in hardware until
// the phase completes (or ~0.5 ms pass) instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(500000u)
      : "memory");
  return ok != 0;
}

// Bounded wait, slow path: returns false if the CTA is aborting or the time limit expired.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, int where,
                                            bool honor_abort) {
  const uint64_t start = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (honor_abort && *abort_flag) return false;
    if (global_ns() - start > kWaitLimitNs) {
      *abort_flag = 1;
      if (atomicCAS(&g_device_status, 0, NNB_E_DEVICE) == 0) g_device_status_where = where;
      return false;
    }
  }
}

// Bounded wait: one inline try_wait (the common, already-completed or soon-completed case) and the
// out-of-line timed loop otherwise.  Keeping the fast path free of calls matters on the MMA-issuing
// thread: a tcgen05.mma holds the issuing thread for its whole issue slot, so anything between two
// K-steps' MMAs (calls, descriptor arithmetic) adds to every step.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int where,
                                          bool honor_abort = true) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag, where, honor_abort);
}

__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint32_t to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

// 32 consecutive TMEM columns of this thread's lane <- 0 (waits for the store).
__device__ __forceinline__ void tmem_zero32(uint32_t taddr) {
  const uint32_t z = 0;
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, "
      "%1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1, %1};" ::"r"(taddr),
      "r"(z)
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// `sbo` bytes apart (a multiple of 128), Blackwell descriptor version 1, base
// offset 0.  The swizzle is a function of the shared-memory address bits
// (measured on B200: a start at any 128-byte row and any multiple-of-128 group
// stride read exactly the rows a TMA box or a row%8-swizzled store wrote from
// a 1024-byte aligned base), so an operand may start inside a swizzle atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t sbo = 1024) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);         // start address   [0,14)
  d |= (uint64_t)1 << 16;                          // LBO (unused for swizzled K-major) [16,30)
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;      // SBO             [32,46)
  d |= (uint64_t)1 << 46;                          // version = 1     [46,48)
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B    [61,64)
  return d;
}

// K-major, 64-byte swizzle: 64-byte rows, 8-row groups of 512 bytes (16-byte
// chunk c of row r stored at chunk c ^ ((r >> 1) & 3)), descriptor version 1.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(512 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;  // SWIZZLE_64B
  return d;
}

// Instruction descriptor: D=f32, A=B=tf32, K-major both, N>>3, M>>4.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor: D=f32, A=B=f16, K-major both, N>>3, M>>4.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor: D=f32, A=B=bf16 (kind::f16 with both operand types bf16), K-major both.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}


}  // namespace tc
}  // namespace nnb
