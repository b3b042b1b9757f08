// Tensor-core (tcgen05 / TMEM) implicit-GEMM 3-D convolution for sm_100a.
//
// GEMM view: M = output voxels of one sample (128-row tiles that never
// straddle samples), N = output channels (BN-wide tiles), K = taps x input
// channels, walked in K-steps of one tap x 32 channels.
//
// Data movement per K-step:
//   A (activations, 128 rows x 32 fp32): producer warps gather each row from
//     global memory (zero for padding taps), apply the lazy instance-norm
//     affine + LeakyReLU of the producing layer, split into TF32 hi/lo and
//     write both halves straight into tensor memory with tcgen05.st.  The
//     A operand of tcgen05.mma is read from TMEM, so activations never pass
//     through shared memory.
//   B (weights, BN rows x 32 fp32 per half): one bulk copy (cp.async.bulk)
//     of a pre-swizzled image (nnb_conv3d_pack) into a 128B-swizzled K-major
//     shared-memory stage, completing on the stage's mbarrier.
//   MMA: one thread issues, per 8-channel sub-step, A_hi*B_hi + A_hi*B_lo +
//     A_lo*B_hi (float32-level accuracy) or A*B (single-pass TF32) into a
//     TMEM float32 accumulator, then tcgen05.commit frees the stage.
// Epilogue: the first producer group reads the accumulator (tcgen05.ld),
// writes the output rows, and writes per-tile (sum, M2) instance-norm
// partials per channel.
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
constexpr int BK = 32;             // input channels per K-step (128 bytes of fp32)
constexpr int kGroups = 3;         // producer warp groups (4 warps each)
constexpr int kProducerWarps = 4 * kGroups;
constexpr int kThreads = (kProducerWarps + 1) * 32;
constexpr int kCtrlWarp = kProducerWarps;
constexpr int kTmemCols = 512;
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

template <int BN, bool SPLIT>
struct Cfg {
  static constexpr int kHalves = SPLIT ? 2 : 1;
  static constexpr int kAcols = BK * kHalves;                      // TMEM columns per A stage
  static constexpr int kAccCols = (BN + 31) / 32 * 32;
  static constexpr int kBBytes = BN * 128 * kHalves;               // smem bytes per B stage
  static constexpr int kTmemStages = (kTmemCols - kAccCols) / kAcols;
  static constexpr int kSmemStages = (200 * 1024) / kBBytes;
  static constexpr int S = (kTmemStages < kSmemStages ? kTmemStages : kSmemStages) > 8
                               ? 8
                               : (kTmemStages < kSmemStages ? kTmemStages : kSmemStages);
  // barriers (<=17 x 8 B), TMEM slot, abort flag, reduction scratch (640 B) and
  // per-channel lazy-affine params (2 x 1024 floats)
  static constexpr int kParamBytes = 512 + 640 + 2 * 1024 * 4;
  static constexpr int kSmemBytes = S * kBBytes + 1024 /*alignment slack*/ + kParamBytes;
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

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false if the CTA is aborting or the time limit expired.
__device__ __noinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int where,
                                       bool honor_abort = true) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0) {
      if (honor_abort && *abort_flag) return false;
      if (global_ns() - start > kWaitLimitNs) {
        *abort_flag = 1;
        if (atomicCAS(&g_device_status, 0, NNB_E_DEVICE) == 0) g_device_status_where = where;
        return false;
      }
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
};

template <int BN, bool SPLIT>
__global__ void __launch_bounds__(kThreads, 1) conv3d_tc_kernel(nnb_conv3d_args a, Geometry g) {
  using C = Cfg<BN, SPLIT>;
  constexpr int S = C::S;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-aligned B stages
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* b_stages = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S * C::kBBytes);
  // bars[0..S) full, [S..2S) empty, [2S] acc_full
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* red = reinterpret_cast<float*>(smem + S * C::kBBytes + 512);  // [4][32]
  float* col_mean = red + 4 * 32;                                       // [32]
  float* s_scale = col_mean + 32;                                       // [cin_total <= 1024]
  float* s_shift = s_scale + 1024;                                      // [cin_total <= 1024]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // tile coordinates: blockIdx.x = (b * tps + t) * n_tiles + nt
  const int nt = blockIdx.x % g.n_tiles;
  const int tile = blockIdx.x / g.n_tiles;
  const int t = tile % g.tps;
  const int b = tile / g.tps;
  const int n0 = nt * BN;
  const int64_t ovox = (int64_t)g.OD * g.OH * g.OW;

  const int c0len = a.seg[0].channels;
  const int cin_total = c0len + (a.num_segments > 1 ? a.seg[1].channels : 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&bars[s]), 5);          // 4 producer warps + 1 expect_tx arrival
      mbar_init(smem_u32(&bars[S + s]), 1);      // tcgen05.commit
    }
    mbar_init(smem_u32(&bars[2 * S]), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  // per-sample lazy affine params for this tile's sample
  for (int c = threadIdx.x; c < cin_total; c += blockDim.x) {
    const int sidx = c < c0len ? 0 : 1;
    const int cl = c < c0len ? c : c - c0len;
    const nnb_segment& sg = a.seg[sidx];
    const int cs = sg.channels;
    s_scale[c] = sg.scale ? sg.scale[(int64_t)b * cs + cl] : 1.f;
    s_shift[c] = sg.scale ? sg.shift[(int64_t)b * cs + cl] : 0.f;
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
  const uint32_t tmem_acc = tmem;
  const uint32_t tmem_a0 = tmem + C::kAccCols;

  if (warp == kCtrlWarp) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(BM, BN);
      for (int ks = 0; ks < g.ksteps; ++ks) {
        const int s = ks % S;
        if (!mbar_wait(smem_u32(&bars[s]), (ks / S) & 1, abort_flag, 1)) break;
        fence_after();
        const uint32_t b_hi = smem_u32(b_stages + s * C::kBBytes);
        const uint32_t a_hi = tmem_a0 + s * C::kAcols;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t dh = sw128_desc(b_hi + kk * 32);
          const uint32_t acc = (ks > 0 || kk > 0) ? 1u : 0u;
          mma_tf32_ts(tmem_acc, a_hi + kk * 8, dh, idesc, acc);
          if constexpr (SPLIT) {
            const uint64_t dl = sw128_desc(b_hi + BN * 128 + kk * 32);
            mma_tf32_ts(tmem_acc, a_hi + kk * 8, dl, idesc, 1u);
            mma_tf32_ts(tmem_acc, a_hi + BK + kk * 8, dh, idesc, 1u);
          }
        }
        mma_commit(smem_u32(&bars[S + s]));
      }
      mma_commit(smem_u32(&bars[2 * S]));
    }
    __syncwarp();
  } else {
    // ------------------------- producers -------------------------
    const int grp = warp >> 2;
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const int64_t m = (int64_t)t * BM + row;
    const bool valid = m < ovox;
    const int ox = (int)(m % g.OW), oy = (int)((m / g.OW) % g.OH), oz = (int)(m / ((int64_t)g.OW * g.OH));
    const int bz = oz * g.SD - g.PD, by = oy * g.SH - g.PH, bx = ox * g.SW - g.PW;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const uint8_t* packed = reinterpret_cast<const uint8_t*>(a.packed) + (int64_t)nt * g.ksteps * C::kBBytes;
    const int64_t in_plane = (int64_t)g.ID * g.IH * g.IW;

    for (int ks = grp; ks < g.ksteps; ks += kGroups) {
      const int s = ks % S;
      if (ks >= S) {
        const bool ok = mbar_wait(smem_u32(&bars[S + s]), ((ks / S) - 1) & 1, abort_flag, 2);
        if (!__all_sync(0xffffffffu, ok)) break;  // warp-uniform exit before .sync.aligned ops
        fence_after();  // order the TMEM overwrite after the MMAs that read this stage
      }
      if (q == 0 && lane == 0) {
        const uint32_t full = smem_u32(&bars[s]);
        mbar_arrive_expect_tx(full, C::kBBytes);
        bulk_g2s(smem_u32(b_stages + s * C::kBBytes), packed + (int64_t)ks * C::kBBytes, C::kBBytes, full);
      }
      const int tap = ks / g.nchunk;
      const int chunk = ks - tap * g.nchunk;
      const int kx = tap % g.KW, ky = (tap / g.KW) % g.KH, kz = tap / (g.KW * g.KH);
      const int iz = bz + kz, iy = by + ky, ix = bx + kx;
      const bool inb = valid && iz >= 0 && iz < g.ID && iy >= 0 && iy < g.IH && ix >= 0 && ix < g.IW;
      const int cglob = chunk * BK;
      const bool second = cglob >= c0len;
      const float* sdata = second ? a.seg[1].data : a.seg[0].data;
      const int schan = second ? a.seg[1].channels : a.seg[0].channels;
      const bool lazy = (second ? a.seg[1].scale : a.seg[0].scale) != nullptr;
      const int sleaky = second ? a.seg[1].leaky : a.seg[0].leaky;
      const int cl = cglob - (second ? c0len : 0);
      float v[32];
      if (inb) {
        const float4* src = reinterpret_cast<const float4*>(
            sdata + (((int64_t)b * in_plane + ((int64_t)iz * g.IH + iy) * g.IW + ix) * schan + cl));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 f = __ldg(src + i);
          v[4 * i + 0] = f.x;
          v[4 * i + 1] = f.y;
          v[4 * i + 2] = f.z;
          v[4 * i + 3] = f.w;
        }
        if (lazy) {
          const float* sc = s_scale + cglob;
          const float* sh = s_shift + cglob;
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float y = fmaf(v[i], sc[i], sh[i]);
            v[i] = sleaky ? leaky(y, a.slope) : y;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = 0.f;
      }
      uint32_t hi[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) hi[i] = to_tf32(v[i]);
      __syncwarp();
      const uint32_t a_stage = tmem_a0 + s * C::kAcols + lane_base;
      tmem_st32(a_stage, hi);
      if constexpr (SPLIT) {
        uint32_t lo[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) lo[i] = to_tf32(v[i] - __uint_as_float(hi[i]));
        tmem_st32(a_stage + BK, lo);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bars[s]));
    }

    // ------------------------- epilogue (group 0) -------------------------
    // The MMA thread always commits acc_full (also after an abort), so this
    // wait ends; the loop below runs unconditionally so that the four warps
    // take the same named barriers.
    if (grp == 0) {
      mbar_wait(smem_u32(&bars[2 * S]), 0, abort_flag, 3, /*honor_abort=*/false);
      fence_after();
      {
        const int rows = (int)min((int64_t)BM, ovox - (int64_t)t * BM);
        for (int cc = 0; cc < C::kAccCols / 32; ++cc) {
          float v[32];
          tmem_ld32(tmem_acc + lane_base + cc * 32, v);
          const int nbase = n0 + cc * 32;
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
      }
      fence_before();
    }
  }
  __syncthreads();
  if (warp == kCtrlWarp) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Weight image: [n_tile][kstep][half][BN rows][128 B, 16-byte chunks XOR-swizzled by row%8]
// ---------------------------------------------------------------------------
__global__ void pack_kernel(const float* __restrict__ w, int cout, int kvol, int cin_total, int bn, int halves,
                            int nchunk, int64_t total_words, uint32_t* __restrict__ out) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total_words;
       o += (int64_t)gridDim.x * blockDim.x) {
    // decompose word index
    const int word = (int)(o % 32);               // word within a 128-byte row (physical)
    int64_t r = o / 32;
    const int n = (int)(r % bn);
    r /= bn;
    const int half = (int)(r % halves);
    r /= halves;
    const int ks = (int)(r % ((int64_t)kvol * nchunk));
    const int nt = (int)(r / ((int64_t)kvol * nchunk));
    const int phys_chunk = word >> 2;
    const int logical_chunk = phys_chunk ^ (n & 7);
    const int k = logical_chunk * 4 + (word & 3);  // channel within the 32-channel step
    const int tap = ks / nchunk;
    const int chunk = ks % nchunk;
    const int co = nt * bn + n;
    const int ci = chunk * BK + k;
    float val = 0.f;
    if (co < cout && ci < cin_total) val = w[((int64_t)co * kvol + tap) * cin_total + ci];
    uint32_t hi;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(val));
    uint32_t res = hi;
    if (half == 1) {
      asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(res) : "f"(val - __uint_as_float(hi)));
    }
    out[o] = res;
  }
}

inline int pick_bn(int cout) {
  if (cout <= 32) return 32;
  if (cout <= 64) return 64;
  if (cout <= 128) return 128;
  if (cout % 160 == 0 || cout > 256) return 160;
  return 128;
}

template <int BN, bool SPLIT>
int launch_bn(const nnb_conv3d_args& a, const Geometry& g, cudaStream_t stream) {
  using C = Cfg<BN, SPLIT>;
  auto kern = conv3d_tc_kernel<BN, SPLIT>;
  static bool configured = false;  // per process; the attribute is per function
  if (!configured) {
    NNB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes));
    configured = true;
  }
  const int64_t blocks = (int64_t)a.batch * g.tps * g.n_tiles;
  NNB_REQUIRE(blocks < (1LL << 31), "conv3d: too many tiles");
  kern<<<(unsigned)blocks, kThreads, C::kSmemBytes, stream>>>(a, g);
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

}  // namespace tc

bool conv3d_tc_supported(const nnb_conv3d_args& a) {
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) {
    if (a.seg[s].channels % tc::BK != 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.seg[s].data) & 15) != 0) return false;
    cin_total += a.seg[s].channels;
  }
  if (cin_total > 1024) return false;
  if (a.cout % 16 != 0) return false;
  return a.precision == NNB_PREC_FP32 || a.precision == NNB_PREC_TF32;
}

int64_t conv3d_tc_packed_bytes(int cout, int kvol, int cin_total, int precision) {
  if (cin_total % tc::BK != 0) return 0;
  const int bn = tc::pick_bn(cout);
  const int n_tiles = (cout + bn - 1) / bn;
  const int halves = precision == NNB_PREC_FP32 ? 2 : 1;
  return (int64_t)n_tiles * kvol * (cin_total / tc::BK) * halves * bn * 128;
}

int launch_conv3d_pack(const float* w, int cout, int kvol, int cin_total, int precision, void* packed,
                       cudaStream_t stream) {
  NNB_REQUIRE(cin_total % tc::BK == 0, "conv3d_pack: input channels must be a multiple of %d", tc::BK);
  NNB_REQUIRE(precision == NNB_PREC_FP32 || precision == NNB_PREC_TF32, "conv3d_pack: precision");
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 1023) == 0, "conv3d_pack: image must be 1024-byte aligned");
  const int bn = tc::pick_bn(cout);
  const int n_tiles = (cout + bn - 1) / bn;
  const int halves = precision == NNB_PREC_FP32 ? 2 : 1;
  const int nchunk = cin_total / tc::BK;
  const int64_t words = (int64_t)n_tiles * kvol * nchunk * halves * bn * 32;
  const int blocks = (int)std::min<int64_t>((words + 255) / 256, 148 * 32);
  tc::pack_kernel<<<blocks, 256, 0, stream>>>(w, cout, kvol, cin_total, bn, halves, nchunk, words,
                                              reinterpret_cast<uint32_t*>(packed));
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_conv3d_tc(const nnb_conv3d_args& a, cudaStream_t stream) {
  tc::Geometry g;
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
  const int64_t ovox = (int64_t)g.OD * g.OH * g.OW;
  g.tps = tiles_per_sample(ovox);
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) cin_total += a.seg[s].channels;
  g.nchunk = cin_total / tc::BK;
  g.ksteps = g.KD * g.KH * g.KW * g.nchunk;
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(a.packed) & 1023) == 0, "conv3d: packed weights must be 1024-aligned");
  const int bn = tc::pick_bn(a.cout);
  g.n_tiles = (a.cout + bn - 1) / bn;
  const bool split = a.precision == NNB_PREC_FP32;
  switch (bn) {
    case 32:
      return split ? tc::launch_bn<32, true>(a, g, stream) : tc::launch_bn<32, false>(a, g, stream);
    case 64:
      return split ? tc::launch_bn<64, true>(a, g, stream) : tc::launch_bn<64, false>(a, g, stream);
    case 128:
      return split ? tc::launch_bn<128, true>(a, g, stream) : tc::launch_bn<128, false>(a, g, stream);
    default:
      return split ? tc::launch_bn<160, true>(a, g, stream) : tc::launch_bn<160, false>(a, g, stream);
  }
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
