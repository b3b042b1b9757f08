// Tensor-core (tcgen05 / TMEM) implicit-GEMM 3-D convolution for sm_100a.
//
// GEMM view: M = output voxels of one sample (128-row tiles that never
// straddle samples), N = output channels (BN-wide tiles), K = taps x input
// channels, walked in K-steps of one tap x 32 channels.
//
// Persistent kernel: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...
// Warp roles (9 warps):
//   warps 0-3   producers (one warp per TMEM lane quarter).  For each step a producer
//               thread gathers its row (one output voxel, 32 input channels;
//               zero for padding taps), applies the lazy instance-norm affine
//               + LeakyReLU of the producing layer, splits it into TF32 hi/lo
//               and writes both halves into a TMEM A stage with tcgen05.st.
//               The gathers of the next two steps are in flight while the
//               current step is transformed and stored.  The group's first thread also issues the bulk copy
//               (cp.async.bulk) of the step's pre-swizzled weight tile into a
//               128B-swizzled K-major shared-memory stage.
//   warp 8      allocates TMEM and issues tcgen05.mma (A from TMEM, B from
//               shared memory): per 8-channel sub-step A_hi*B_hi + A_hi*B_lo +
//               A_lo*B_hi (float32-level accuracy) or A*B (single-pass TF32),
//               into one of two TMEM accumulators; tcgen05.commit releases the
//               stage and, after the tile's last step, the accumulator.
//   warps 4-7   epilogue: tcgen05.ld of a finished accumulator (overlapping
//               the next tile's main loop), output rows to global memory and
//               per-tile (sum, M2) instance-norm partials, or -- for a
//               stride == kernel transposed convolution -- the scatter of each
//               (tap, channel) column block to its up-sampled voxel plus bias.
//
// Every mbarrier wait is bounded by the global timer; on expiry the CTA
// records NNB_E_DEVICE in a device status word and drains.
#include <cuda_runtime.h>

#include <algorithm>
#include <stdint.h>

#include "common.cuh"

namespace nnb {

__device__ int g_device_status = 0;      // first device-side error code (0 = ok)
__device__ int g_device_status_where = 0;

namespace tc {

constexpr int BM = 128;
constexpr int BK = 32;              // input channels per K-step (128 bytes of fp32)
constexpr int kProducerWarps = 4;               // one warp per TMEM lane quarter
constexpr int kCtrlWarp = kProducerWarps + 4;    // warps 4..7 epilogue, warp 8 MMA
constexpr int kThreads = (kCtrlWarp + 1) * 32;
constexpr int kTmemCols = 512;
constexpr int kMaxSmem = 227 * 1024;
constexpr int kMaxKsteps = 1024;                 // K-step table capacity (taps x 32-channel chunks)
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

template <int BN, bool SPLIT>
struct Cfg {
  static constexpr int kHalves = SPLIT ? 2 : 1;
  static constexpr int kAcols = BK * kHalves;                      // TMEM columns per A stage
  static constexpr int kAccCols = (BN + 31) / 32 * 32;
  static constexpr int kAccBufs = (2 * kAccCols + 4 * kAcols <= kTmemCols) ? 2 : 1;
  static constexpr int kBBytes = BN * 128 * kHalves;               // smem bytes per B stage
  static constexpr int kTmemStages = (kTmemCols - kAccBufs * kAccCols) / kAcols;
  static constexpr int kSmemStages = (176 * 1024) / kBBytes;
  static constexpr int kS0 = kTmemStages < kSmemStages ? kTmemStages : kSmemStages;
  static constexpr int S = kS0 > 8 ? 8 : kS0;
  // barriers (2S + 4 x 8 B), TMEM slot, abort/vote words, epilogue scratch
  static constexpr int kMiscBytes = 1024;
  static constexpr int kFixedSmem = S * kBBytes + 1024 /*alignment slack*/ + kMiscBytes + 8 * kMaxKsteps;
  static_assert(S >= 2, "too few pipeline stages");
};

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

// Bounded wait: returns false if the CTA is aborting or the time limit expired.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int where,
                                       bool honor_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
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

// 32 consecutive TMEM columns of this thread's lane <- v[0..31]
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// 16 TMEM lanes x 32 columns from a warp: register k of thread t goes to lane
// taddr.lane + t/4 + 8*((k>>1)&1), column taddr.col + 8*(k>>2) + 2*(t%4) + (k&1).
__device__ __forceinline__ void tmem_st16x256_x4(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
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
// 1024 bytes apart (SBO), Blackwell descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);         // start address   [0,14)
  d |= (uint64_t)1 << 16;                          // LBO (unused for swizzled K-major) [16,30)
  d |= (uint64_t)(1024 >> 4) << 32;                // SBO             [32,46)
  d |= (uint64_t)1 << 46;                          // version = 1     [46,48)
  d |= (uint64_t)2 << 61;                          // SWIZZLE_128B    [61,64)
  return d;
}

// Instruction descriptor: D=f32, A=B=tf32, K-major both, N>>3, M>>4.
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// Transpose-reduce: lane j ends with sum over the warp's lanes of x[j].
__device__ __forceinline__ float warp_column_sums(float (&x)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int h = 16; h >= 1; h >>= 1) {
    const bool up = (lane & h) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = up ? x[i] : x[i + h];
      const float keep = up ? x[i + h] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, h);
    }
  }
  return x[0];
}

struct Geometry {
  int ID, IH, IW, OD, OH, OW;
  int KD, KH, KW, SD, SH, SW, PD, PH, PW;
  int tps;          // tiles per sample
  int nchunk;       // 32-channel chunks over all segments
  int ksteps;       // taps * nchunk
  int n_tiles;      // N tiles
  int total_tiles;  // batch * tps * n_tiles
  int cin_total;
  // scatter epilogue (stride == kernel transposed convolution); up_cout == 0 for a convolution
  int up_cout, UKD, UKH, UKW;
};

// Per-thread row state of the tile currently being gathered (recomputed only
// when the tile changes).  A producer thread owns rows t/4 + 8i (i = 0..3) of
// its warp's lane quarter: for each, the linear index of the voxel that tap 0
// reads ((b, z, y, x) of the window corner, possibly outside the volume) and a
// bit mask of the taps that fall inside the input.
struct RowState {
  int it, nt;
  int64_t corner[4];
  uint32_t taps[4];
};

__device__ __forceinline__ void row_state_update(const Geometry& g, int it, int qrow0, RowState& rs) {
  const int tile = blockIdx.x + it * gridDim.x;
  const int mt = tile / g.n_tiles;
  const int t = mt % g.tps;
  const int b = mt / g.tps;
  const int64_t ovox = (int64_t)g.OD * g.OH * g.OW;
  rs.it = it;
  rs.nt = tile - mt * g.n_tiles;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = (int64_t)t * BM + qrow0 + 8 * i;
    uint32_t mask = 0;
    int64_t corner = 0;
    if (m < ovox) {
      const int ox = (int)(m % g.OW), oy = (int)((m / g.OW) % g.OH), oz = (int)(m / ((int64_t)g.OW * g.OH));
      const int bz = oz * g.SD - g.PD, by = oy * g.SH - g.PH, bx = ox * g.SW - g.PW;
      corner = (((int64_t)b * g.ID + bz) * g.IH + by) * g.IW + bx;
      int tap = 0;
      for (int kz = 0; kz < g.KD; ++kz) {
        const bool okz = bz + kz >= 0 && bz + kz < g.ID;
        for (int ky = 0; ky < g.KH; ++ky) {
          const bool oky = okz && by + ky >= 0 && by + ky < g.IH;
          for (int kx = 0; kx < g.KW; ++kx, ++tap) {
            if (oky && bx + kx >= 0 && bx + kx < g.IW) mask |= 1u << tap;
          }
        }
      }
    }
    rs.corner[i] = corner;
    rs.taps[i] = mask;
  }
}

// One half-step of a thread: rows 2h and 2h+1, 8 channels each, hi (and lo).
struct HalfInfo {
  int it, ks, nt;
};

// K-step table entry: .x = tap | chunk << 8, .y = voxel offset of the tap from the window corner
template <bool SPLIT>
__device__ __forceinline__ void gather_half(const nnb_conv3d_args& a, const Geometry& g, int it, int ks, int half,
                                            int qrow0, int cq, const int2* kstab, RowState& rs, HalfInfo& info,
                                            float (&v)[32]) {
  if (it != rs.it) row_state_update(g, it, qrow0, rs);
  const int2 e = kstab[ks];
  const int tap = e.x & 255;
  const int cglob = (e.x >> 8) * BK;
  const bool second = cglob >= a.seg[0].channels;
  const float* sdata = second ? a.seg[1].data : a.seg[0].data;
  const int schan = second ? a.seg[1].channels : a.seg[0].channels;
  const int cl = cglob - (second ? a.seg[0].channels : 0) + 8 * cq;
  const int64_t rstride = (int64_t)(SPLIT ? 2 : 1) * schan;  // floats per voxel of the prepared operand
  info.it = it;
  info.ks = ks;
  info.nt = rs.nt;
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int i = 2 * half + j;
    if ((rs.taps[i] >> tap) & 1u) {
      const float* src = sdata + (rs.corner[i] + e.y) * rstride + cl;
      const float4 h0 = __ldg(reinterpret_cast<const float4*>(src));
      const float4 h1 = __ldg(reinterpret_cast<const float4*>(src) + 1);
      v[16 * j + 0] = h0.x; v[16 * j + 1] = h0.y; v[16 * j + 2] = h0.z; v[16 * j + 3] = h0.w;
      v[16 * j + 4] = h1.x; v[16 * j + 5] = h1.y; v[16 * j + 6] = h1.z; v[16 * j + 7] = h1.w;
      if constexpr (SPLIT) {
        const float4 l0 = __ldg(reinterpret_cast<const float4*>(src + schan));
        const float4 l1 = __ldg(reinterpret_cast<const float4*>(src + schan) + 1);
        v[16 * j + 8] = l0.x; v[16 * j + 9] = l0.y; v[16 * j + 10] = l0.z; v[16 * j + 11] = l0.w;
        v[16 * j + 12] = l1.x; v[16 * j + 13] = l1.y; v[16 * j + 14] = l1.z; v[16 * j + 15] = l1.w;
      }
    } else {
#pragma unroll
      for (int f = 0; f < 16; ++f) v[16 * j + f] = 0.f;
    }
  }
}

// Registers of one 16x256b.x4 store from two rows' 8 values: register k -> lane
// +8*((k>>1)&1), column 8*(k>>2) + 2*(t%4) + (k&1); TMEM column 8*rep + 2*(t%4) + e
// holds channel 8*(t%4) + 2*rep + e (the weight image uses the same K order).
__device__ __forceinline__ void st_rows(uint32_t taddr, const float (&v)[32], int off) {
  uint32_t r[16];
#pragma unroll
  for (int rep = 0; rep < 4; ++rep) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      r[4 * rep + e] = __float_as_uint(v[off + 2 * rep + e]);
      r[4 * rep + 2 + e] = __float_as_uint(v[16 + off + 2 * rep + e]);
    }
  }
  tmem_st16x256_x4(taddr, r);
}

// Returns false when the CTA is aborting.
template <int BN, bool SPLIT>
__device__ __forceinline__ bool process_half(const nnb_conv3d_args& a, const Geometry& g, int G, int half,
                                             const HalfInfo& info, const float (&v)[32], uint64_t* bars,
                                             uint8_t* b_stages, uint32_t tmem_a0, uint32_t lane_base, bool leader,
                                             volatile int* abort_flag, int& s) {
  using C = Cfg<BN, SPLIT>;
  constexpr int S = C::S;
  if (half == 0) {
    if (G >= S) {
      const bool ok = mbar_wait(smem_u32(&bars[S + s]), ((G / S) - 1) & 1, abort_flag, 2);
      if (!__all_sync(0xffffffffu, ok)) return false;  // warp-uniform exit before .sync.aligned ops
      fence_after();  // order the TMEM overwrite after the MMAs that read this stage
    }
    if (leader) {
      const uint8_t* src = reinterpret_cast<const uint8_t*>(a.packed) +
                           ((int64_t)info.nt * g.ksteps + info.ks) * C::kBBytes;
      const uint32_t full = smem_u32(&bars[s]);
      mbar_arrive_expect_tx(full, C::kBBytes);
      bulk_g2s(smem_u32(b_stages + s * C::kBBytes), src, C::kBBytes, full);
    }
  }
  __syncwarp();
  const uint32_t a_stage = tmem_a0 + s * C::kAcols + lane_base + ((16u * half) << 16);
  st_rows(a_stage, v, 0);
  if constexpr (SPLIT) st_rows(a_stage + BK, v, 8);
  if (half == 1) {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
    fence_before();
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&bars[s]));
    if (++s == S) s = 0;
  }
  return true;
}

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) conv3d_tc_kernel(nnb_conv3d_args a, Geometry g) {
  using C = Cfg<BN, SPLIT>;
  constexpr int S = C::S;
  constexpr int NB = C::kAccBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = smem;
  uint8_t* misc = smem + S * C::kBBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc);  // full[S], empty[S], accf[2], acce[2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 8 * (2 * S + 4));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* votes = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [4]
  float* red = reinterpret_cast<float*>(misc + 256);                      // [4][32]
  float* col_mean = red + 4 * 32;                                         // [32]
  int2* kstab = reinterpret_cast<int2*>(misc + C::kMiscBytes);            // [ksteps <= kMaxKsteps]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int my_tiles = (g.total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int64_t ovox = (int64_t)g.OD * g.OH * g.OW;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&bars[s]), 5);      // 4 producer warps + 1 expect_tx arrival
      mbar_init(smem_u32(&bars[S + s]), 1);  // tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&bars[2 * S + i]), 1);      // accumulator full: tcgen05.commit
      mbar_init(smem_u32(&bars[2 * S + 2 + i]), 4);  // accumulator empty: 4 epilogue warps
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  for (int ks = threadIdx.x; ks < g.ksteps; ks += blockDim.x) {
    const int tap = ks / g.nchunk, chunk = ks - tap * g.nchunk;
    const int kx = tap % g.KW, ky = (tap / g.KW) % g.KH, kz = tap / (g.KW * g.KH);
    kstab[ks] = make_int2(tap | (chunk << 8), (kz * g.IH + ky) * g.IW + kx);
  }
  if (warp == kCtrlWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tmem_a0 = tmem + NB * C::kAccCols;

  if (warp == kCtrlWarp) {
    // ------------------------------ MMA issuer ------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      bool alive = true;
      for (int it = 0; it < my_tiles && alive; ++it) {
        const int ab = NB == 2 ? (it & 1) : 0;
        if (it >= NB) {
          if (!mbar_wait(smem_u32(&bars[2 * S + 2 + ab]), ((it / NB) - 1) & 1, abort_flag, 4)) break;
          fence_after();
        }
        const uint32_t d = tmem + ab * C::kAccCols;
        for (int ks = 0; ks < g.ksteps; ++ks) {
          const int G = it * g.ksteps + ks;
          const int s = G % S;
          if (!mbar_wait(smem_u32(&bars[s]), (G / S) & 1, abort_flag, 1)) {
            alive = false;
            break;
          }
          fence_after();
          const uint32_t b_hi = smem_u32(b_stages + s * C::kBBytes);
          const uint32_t a_hi = tmem_a0 + s * C::kAcols;
#pragma unroll
          for (int kk = 0; kk < BK / 8; ++kk) {
            const uint64_t dh = sw128_desc(b_hi + kk * 32);
            mma_tf32_ts(d, a_hi + kk * 8, dh, idesc, (ks > 0 || kk > 0) ? 1u : 0u);
            if constexpr (SPLIT) {
              const uint64_t dl = sw128_desc(b_hi + BN * 128 + kk * 32);
              mma_tf32_ts(d, a_hi + kk * 8, dl, idesc, 1u);
              mma_tf32_ts(d, a_hi + BK + kk * 8, dh, idesc, 1u);
            }
          }
          mma_commit(smem_u32(&bars[S + s]));
        }
        mma_commit(smem_u32(&bars[2 * S + ab]));
      }
    }
    __syncwarp();
  } else if (warp < kProducerWarps) {
    // ------------------------------ producers -------------------------------
    const int q = warp & 3;
    const int qrow0 = q * 32 + (lane >> 2);  // first of this thread's rows (then +8, +16, +24)
    const int cq = lane & 3;                 // 8-channel group of this thread
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const bool leader = (q == 0 && lane == 0);
    // Half-steps H = 2G + half: three register buffers keep the gathers of the
    // next two half-steps in flight while the current one is stored to TMEM.
    const int total = 2 * my_tiles * g.ksteps;
    RowState rs;
    rs.it = -1;
    int pit = 0, pks = 0, phalf = 0;  // next half-step to gather
    auto gather_next = [&](HalfInfo& info, float (&v)[32]) {
      gather_half<SPLIT>(a, g, pit, pks, phalf, qrow0, cq, kstab, rs, info, v);
      if (++phalf == 2) {
        phalf = 0;
        if (++pks == g.ksteps) {
          pks = 0;
          ++pit;
        }
      }
    };
    HalfInfo i0, i1, i2;
    float v0[32], v1[32], v2[32];
    int H = 0;
    int stage = 0;
    if (total > 0) gather_next(i0, v0);
    if (total > 1) gather_next(i1, v1);
    while (H < total) {
      if (H + 2 < total) gather_next(i2, v2);
      if (!process_half<BN, SPLIT>(a, g, H >> 1, H & 1, i0, v0, bars, b_stages, tmem_a0, lane_base, leader,
                                   abort_flag, stage))
        break;
      if (++H >= total) break;
      if (H + 2 < total) gather_next(i0, v0);
      if (!process_half<BN, SPLIT>(a, g, H >> 1, H & 1, i1, v1, bars, b_stages, tmem_a0, lane_base, leader,
                                   abort_flag, stage))
        break;
      if (++H >= total) break;
      if (H + 2 < total) gather_next(i1, v1);
      if (!process_half<BN, SPLIT>(a, g, H >> 1, H & 1, i2, v2, bars, b_stages, tmem_a0, lane_base, leader,
                                   abort_flag, stage))
        break;
      ++H;
    }
  } else {
    // ------------------------------ epilogue ---------------------------------
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const int row = q * 32 + lane;
    for (int it = 0; it < my_tiles; ++it) {
      const int ab = NB == 2 ? (it & 1) : 0;
      const bool ok = mbar_wait(smem_u32(&bars[2 * S + ab]), (it / NB) & 1, abort_flag, 3);
      // consistent stop decision across the four epilogue warps
      if (lane == 0) votes[q] = (!ok || *abort_flag) ? 1 : 0;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const bool stop = votes[0] | votes[1] | votes[2] | votes[3];
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (stop) break;
      fence_after();
      const int tile = blockIdx.x + it * gridDim.x;
      const int nt = tile % g.n_tiles;
      const int mt = tile / g.n_tiles;
      const int t = mt % g.tps;
      const int b = mt / g.tps;
      const int64_t m = (int64_t)t * BM + row;
      const bool valid = m < ovox;
      const int rows = (int)min((int64_t)BM, ovox - (int64_t)t * BM);
      const int n0 = nt * BN;
      const uint32_t acc = tmem + ab * C::kAccCols + lane_base;
      for (int cc = 0; cc < C::kAccCols / 32; ++cc) {
        float v[32];
        tmem_ld32(acc + cc * 32, v);
        const int nbase = n0 + cc * 32;
        if (nbase >= a.cout) continue;  // uniform: whole chunk beyond N
        if (g.up_cout > 0) {
          // scatter: column n = tap * up_cout + co of input voxel m -> up-sampled voxel
          const int tap = nbase / g.up_cout;
          const int co0 = nbase - tap * g.up_cout;
          if (valid) {
            const int ux = tap % g.UKW, uy = (tap / g.UKW) % g.UKH, uz = tap / (g.UKW * g.UKH);
            const int ix = (int)(m % g.OW), iy = (int)((m / g.OW) % g.OH), iz = (int)(m / ((int64_t)g.OW * g.OH));
            const int OD2 = g.OD * g.UKD, OH2 = g.OH * g.UKH, OW2 = g.OW * g.UKW;
            float* dst = a.out + ((((int64_t)b * OD2 + iz * g.UKD + uz) * OH2 + iy * g.UKH + uy) * OW2 +
                                  ix * g.UKW + ux) * g.up_cout + co0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (a.bias != nullptr) v[i] += __ldg(a.bias + co0 + i);
#pragma unroll
            for (int i = 0; i < 8; ++i)
              reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
          continue;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int n = nbase + i;
          if (a.bias != nullptr && n < a.cout) v[i] += __ldg(a.bias + n);
          if (!valid) v[i] = 0.f;
        }
        if (valid) {
          float* dst = a.out + ((int64_t)b * ovox + m) * a.cout + nbase;
          if (nbase + 32 <= a.cout && (a.cout % 4) == 0) {
#pragma unroll
            for (int i = 0; i < 8; ++i)
              reinterpret_cast<float4*>(dst)[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (nbase + i < a.cout) dst[i] = v[i];
          }
        }
        if (a.partials != nullptr) {
          float x[32];
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = v[i];
          const float colsum = warp_column_sums(x);
          red[q * 32 + lane] = colsum;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (q == 0) col_mean[lane] = (red[lane] + red[32 + lane] + red[64 + lane] + red[96 + lane]) / rows;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          const float total = red[lane] + red[32 + lane] + red[64 + lane] + red[96 + lane];
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float d = valid ? v[i] - col_mean[i] : 0.f;
            x[i] = d * d;
          }
          const float colm2 = warp_column_sums(x);
          asm volatile("bar.sync 1, 128;" ::: "memory");
          red[q * 32 + lane] = colm2;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (q == 0 && nbase + lane < a.cout) {
            const float m2 = red[lane] + red[32 + lane] + red[64 + lane] + red[96 + lane];
            float* p = a.partials + (((int64_t)b * g.tps + t) * a.cout + nbase + lane) * 2;
            p[0] = total;
            p[1] = m2;
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
        }
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[2 * S + 2 + ab]));
    }
  }
  __syncthreads();
  if (warp == kCtrlWarp) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Weight image: [n_tile][kstep][half][BN rows][128 B, 16-byte chunks XOR-swizzled by row%8].
// GEMM row n of a convolution is output channel n; for a transposed
// convolution (row_taps > 1) row n is (tap = n / up_cout, channel = n % up_cout)
// and the single K tap reads weight (channel, tap, ci).
// ---------------------------------------------------------------------------
__global__ void pack_kernel(const float* __restrict__ w, int rows_total, int kvol, int cin_total, int bn, int halves,
                            int nchunk, int row_taps, int up_cout, int64_t total_words, uint32_t* __restrict__ out) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total_words;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int word = (int)(o % 32);  // 4-byte word within a 128-byte row (physical position)
    int64_t r = o / 32;
    const int n = (int)(r % bn);
    r /= bn;
    const int half = (int)(r % halves);
    r /= halves;
    const int ks = (int)(r % ((int64_t)kvol * nchunk));
    const int nt = (int)(r / ((int64_t)kvol * nchunk));
    const int logical_chunk = (word >> 2) ^ (n & 7);
    const int c = logical_chunk * 4 + (word & 3);  // K column within the 32-channel step
    // K column 8*rep + 2*j + e holds channel 8*j + 2*rep + e (the A operand's TMEM order)
    const int k = 8 * ((c & 7) >> 1) + 2 * (c >> 3) + (c & 1);
    const int tap = ks / nchunk;
    const int chunk = ks % nchunk;
    const int row = nt * bn + n;
    const int ci = chunk * BK + k;
    float val = 0.f;
    if (row < rows_total && ci < cin_total) {
      if (row_taps > 1) {
        const int co = row % up_cout, utap = row / up_cout;
        val = w[((int64_t)co * row_taps + utap) * cin_total + ci];
      } else {
        val = w[((int64_t)row * kvol + tap) * cin_total + ci];
      }
    }
    uint32_t res;
    if (halves == 2) {
      const uint32_t hi = __float_as_uint(val) & 0xFFFFE000u;
      res = half == 0 ? hi : __float_as_uint(val - __uint_as_float(hi));
    } else {
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(res) : "f"(val));
    }
    out[o] = res;
  }
}

inline int pick_bn(int n) {
  if (n <= 32) return 32;
  if (n <= 64) return 64;
  if (n % 128 == 0 || n <= 128) return 128;
  if (n % 160 == 0) return 160;
  return 128;
}

template <int BN, bool SPLIT>
int launch_bn(const nnb_conv3d_args& a, Geometry g, cudaStream_t stream) {
  using C = Cfg<BN, SPLIT>;
  auto kern = conv3d_tc_kernel<BN, SPLIT>;
  const int smem = C::kFixedSmem;
  int dev = 0;
  NNB_CUDA_CHECK(cudaGetDevice(&dev));
  static int configured_max[64] = {0};  // largest dynamic smem set per device for this instantiation
  if (dev < 64 && configured_max[dev] < smem) {
    NNB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    configured_max[dev] = kMaxSmem;
  }
  int sms = 148;
  NNB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::min(g.total_tiles, sms);
  kern<<<grid, kThreads, smem, stream>>>(a, g);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int dispatch(const nnb_conv3d_args& a, Geometry& g, cudaStream_t stream) {
  const int bn = pick_bn(a.cout);
  g.n_tiles = (a.cout + bn - 1) / bn;
  const int64_t tiles = (int64_t)a.batch * g.tps * g.n_tiles;
  NNB_REQUIRE(tiles < (1LL << 31), "conv3d: too many tiles");
  g.total_tiles = (int)tiles;
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(a.packed) & 1023) == 0, "conv3d: packed weights must be 1024-aligned");
  const bool split = a.precision == NNB_PREC_FP32;
  switch (bn) {
    case 32:
      return split ? launch_bn<32, true>(a, g, stream) : launch_bn<32, false>(a, g, stream);
    case 64:
      return split ? launch_bn<64, true>(a, g, stream) : launch_bn<64, false>(a, g, stream);
    case 128:
      return split ? launch_bn<128, true>(a, g, stream) : launch_bn<128, false>(a, g, stream);
    default:
      return split ? launch_bn<160, true>(a, g, stream) : launch_bn<160, false>(a, g, stream);
  }
}

Geometry base_geometry(const nnb_conv3d_args& a) {
  Geometry g{};
  g.ID = a.in_dims[0];
  g.IH = a.in_dims[1];
  g.IW = a.in_dims[2];
  g.OD = a.out_dims[0];
  g.OH = a.out_dims[1];
  g.OW = a.out_dims[2];
  g.KD = a.kernel[0];
  g.KH = a.kernel[1];
  g.KW = a.kernel[2];
  g.SD = a.stride[0];
  g.SH = a.stride[1];
  g.SW = a.stride[2];
  g.PD = a.pad[0];
  g.PH = a.pad[1];
  g.PW = a.pad[2];
  g.tps = tiles_per_sample((int64_t)g.OD * g.OH * g.OW);
  g.cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) g.cin_total += a.seg[s].channels;
  g.nchunk = g.cin_total / BK;
  g.ksteps = g.KD * g.KH * g.KW * g.nchunk;
  return g;
}

}  // namespace tc

bool conv3d_tc_supported(const nnb_conv3d_args& a) {
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) {
    if (a.seg[s].channels % tc::BK != 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.seg[s].data) & 15) != 0) return false;
    cin_total += a.seg[s].channels;
  }
  if (a.cout % 16 != 0) return false;
  // K-step table: taps x chunks entries, tap offsets < 16 per axis, chunk index < 2^19
  if ((int64_t)a.kernel[0] * a.kernel[1] * a.kernel[2] * (cin_total / tc::BK) > tc::kMaxKsteps) return false;
  if (a.kernel[0] > 15 || a.kernel[1] > 15 || a.kernel[2] > 15) return false;
  return a.precision == NNB_PREC_FP32 || a.precision == NNB_PREC_TF32;
}

int64_t conv3d_tc_packed_bytes(int rows, int kvol, int cin_total, int precision) {
  if (cin_total % tc::BK != 0) return 0;
  const int bn = tc::pick_bn(rows);
  const int n_tiles = (rows + bn - 1) / bn;
  const int halves = precision == NNB_PREC_FP32 ? 2 : 1;
  return (int64_t)n_tiles * kvol * (cin_total / tc::BK) * halves * bn * 128;
}

int launch_conv3d_pack_rows(const float* w, int rows, int kvol, int cin_total, int precision, int row_taps,
                            int up_cout, void* packed, cudaStream_t stream) {
  NNB_REQUIRE(cin_total % tc::BK == 0, "pack: input channels must be a multiple of %d", tc::BK);
  NNB_REQUIRE(precision == NNB_PREC_FP32 || precision == NNB_PREC_TF32, "pack: precision");
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 1023) == 0, "pack: image must be 1024-byte aligned");
  const int bn = tc::pick_bn(rows);
  const int n_tiles = (rows + bn - 1) / bn;
  const int halves = precision == NNB_PREC_FP32 ? 2 : 1;
  const int nchunk = cin_total / tc::BK;
  const int64_t words = (int64_t)n_tiles * kvol * nchunk * halves * bn * 32;
  const int blocks = (int)std::min<int64_t>((words + 255) / 256, 148 * 32);
  tc::pack_kernel<<<blocks, 256, 0, stream>>>(w, rows, kvol, cin_total, bn, halves, nchunk, row_taps, up_cout, words,
                                              reinterpret_cast<uint32_t*>(packed));
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_conv3d_pack(const float* w, int cout, int kvol, int cin_total, int precision, void* packed,
                       cudaStream_t stream) {
  return launch_conv3d_pack_rows(w, cout, kvol, cin_total, precision, 1, cout, packed, stream);
}

int launch_conv3d_tc(const nnb_conv3d_args& a, cudaStream_t stream) {
  tc::Geometry g = tc::base_geometry(a);
  g.up_cout = 0;
  return tc::dispatch(a, g, stream);
}

// Stride == kernel transposed convolution as a 1x1x1 GEMM (rows = input
// voxels, N = taps x cout) with the scatter epilogue.
int launch_conv_transpose_tc(const nnb_segment& in, int batch, const int32_t in_dims[3], const int32_t k[3],
                             float slope, const float* bias, int cout, const void* packed, int precision, float* out,
                             cudaStream_t stream) {
  nnb_conv3d_args a{};
  a.batch = batch;
  for (int i = 0; i < 3; ++i) {
    a.in_dims[i] = in_dims[i];
    a.out_dims[i] = in_dims[i];
    a.kernel[i] = 1;
    a.stride[i] = 1;
    a.pad[i] = 0;
  }
  a.num_segments = 1;
  a.seg[0] = in;
  a.slope = slope;
  a.cout = cout * k[0] * k[1] * k[2];
  a.weight = nullptr;
  a.packed = packed;
  a.bias = bias;
  a.out = out;
  a.partials = nullptr;
  a.precision = precision;
  a.operand_format = 1;
  NNB_REQUIRE(in.scale == nullptr, "conv_transpose3d: prepared operands carry no lazy affine");
  NNB_REQUIRE(conv3d_tc_supported(a) && cout % 32 == 0, "conv_transpose3d: outside the tensor-core envelope");
  tc::Geometry g = tc::base_geometry(a);
  g.up_cout = cout;
  g.UKD = k[0];
  g.UKH = k[1];
  g.UKW = k[2];
  return tc::dispatch(a, g, stream);
}

}  // namespace nnb

extern "C" int32_t nnb_device_status(int32_t* where, int32_t reset) {
  int status = 0, loc = 0;
  if (cudaMemcpyFromSymbol(&status, nnb::g_device_status, sizeof(int)) != cudaSuccess) return NNB_E_CUDA;
  cudaMemcpyFromSymbol(&loc, nnb::g_device_status_where, sizeof(int));
  if (where) *where = loc;
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(nnb::g_device_status, &zero, sizeof(int));
    cudaMemcpyToSymbol(nnb::g_device_status_where, &zero, sizeof(int));
  }
  return status;
}
