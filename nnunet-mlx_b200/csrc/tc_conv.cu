// Tensor-core (tcgen05 / TMEM / TMA) implicit-GEMM 3-D convolution for sm_100a.
//
// GEMM view: M = output voxels of one sample, N = output channels, K = taps x
// input channels, walked in steps of 32 channels.  Operands are prepared once
// per activation by nnb_prepare_operand (the producing layer's instance-norm
// affine + LeakyReLU applied, converted to the MMA's operand format), so no
// thread touches activations in the main loop.  Operand formats (template OP):
//
//  * kOperandF16x2 (float32-level accuracy, the default): per 32 channels one
//    128-byte row [hi(32) | lo(32)] of halves, x ~ hi + lo (lo = fp16(x - hi),
//    subnormal for small x, whose absolute error then stays below 2^-25).  B
//    stacks [W0 ; W1] along N (W0 = fp16(s w), W1 = fp16(s w - W0), s a power
//    of two per output column), so per 16-channel sub-step A_hi x [W0;W1]
//    (N = 2 BC) and A_lo x W0 (N = BC, into the second half) form the three
//    leading products in two MMAs of kind::f16; the epilogue returns
//    (D0 + D1) / s.
//  * kOperandTf32x2 (split TF32, any float32 magnitude): A hi and lo rows of 32
//    TF32 values, B = [W_hi ; W_lo]; per 8-channel sub-step A_hi x [W_hi;W_lo]
//    and A_lo x [W_hi;W_lo]; the epilogue adds the halves.
//  * kOperandTf32 (fast): one TF32 row, B = W_tf32, one MMA per sub-step.
//  * kOperandBf16 (fast): the fp16 pair's 128-byte A row with bf16(x) in the
//    hi half (the lo half is never read), B = bf16(w) in 64-byte rows; one
//    kind::f16 MMA (A and B both bf16, float32 accumulation) per 16-channel
//    sub-step.
//
// A tcgen05.mma costs at least ~46 cycles at M = 128 whatever N is (up to 64),
// so stacking the split weights along N halves the instruction count of the
// 32- and 64-channel layers, and fp16's 16-channel K per instruction halves it
// again relative to TF32.
//
// Two ways to feed A, both from tiled TMA box loads (5-D map (channels, W, H,
// D, batch), 128-byte swizzle, zero fill outside the volume = the padding):
//
//  * halo mode (stride 1, taps > 1, <= 64 output channels per tile): a tile is
//    an 8 (w) x 16 (h) brick of output voxels.  Per (32-channel chunk, kz) one
//    box brings the (8+KW-1) x (16+KH-1) input plane the brick's taps of that
//    kz read; the MMA of tap (kx, ky) reads it through a descriptor starting
//    (ky * pw + kx) rows in with 8-row groups pw rows apart (pw = 8+KW-1).  The
//    128B swizzle is a function of the shared-memory address, so such
//    unaligned starts and strides read exactly the rows the box wrote.  A
//    3x3x3 conv then loads 3 planes of 180 rows per chunk instead of 27 boxes
//    of 128 rows.  B streams per tap through its own ring.
//  * box mode (everything else: strided convs, 1x1x1 GEMMs, wide layers):
//    the tile is a brick chosen to cover the volume with the fewest tiles and
//    each K-step (one tap x 32 channels) loads one box per half, the brick
//    shifted by the tap offset and sampled every stride voxels (element
//    strides = conv strides), plus that step's B tile.
//
// Persistent kernel, one CTA per SM walking tiles blockIdx.x, +gridDim.x, ...
//   warp 0      one thread issues the TMA box loads and the B bulk copies.
//   warp 1      allocates TMEM; one thread issues tcgen05.mma into one of two
//               TMEM accumulators and tcgen05.commit releases stages and
//               finished accumulators.
//   warps 2-5   epilogue: tcgen05.ld of a finished accumulator (overlapping the
//               next tile's main loop), bias, output rows, per-tile
//               (sum, M2, n) instance-norm partials -- or, for a stride ==
//               kernel transposed convolution run as a 1x1x1 GEMM with
//               N = taps x channels, the scatter of each (tap, channel) block
//               to its up-sampled voxel.
//
// Every mbarrier wait is bounded by the global timer; on expiry the CTA
// records NNB_E_DEVICE in a device status word, waits (bounded) for its
// copies and MMAs in flight, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <stdint.h>

#include "common.cuh"

namespace nnb {
__device__ int g_device_status = 0;
__device__ int g_device_status_where = 0;
}  // namespace nnb

#include "tc_common.cuh"
#include "zs_schedule.cuh"

namespace nnb {
namespace tc {

constexpr int kMiscBytes = 2048;  // mbarriers, TMEM slot, flags, stop votes
constexpr int kMaxBars = 48;
constexpr int kStagingBytes = 2048;  // per epilogue warp: 16 output rows of 32 floats (coalesced stores)
constexpr int kStageBudget = kMaxSmem - 1024 /*alignment slack*/ - kMiscBytes - 4 * kMaxKsteps - 8 * kStagingBytes;
constexpr int kHaloW = 8;   // halo-mode brick: 8 (w) x 16 (h) x 1 (d)
constexpr int kHaloH = 16;

struct Geometry {
  int ID, IH, IW;        // input volume (tensor map extent)
  int OD, OH, OW;        // GEMM row space: output voxels (input voxels for a transposed conv)
  int KD, KH, KW, SD, SH, SW, PD, PH, PW;
  int tw, th, td, rows;  // brick of one tile, rows = tw * th * td <= 128
  int nw, nh, tps;       // bricks along w and h; bricks per sample
  int n_tiles, total_tiles;
  int nchunk, ksteps, c0len;
  int up_cout, UKD, UKH, UKW;  // transposed convolution scatter (up_cout = 0 otherwise)
  int up_operand;              // 1: the scatter writes the fp16-pair operand rows instead of float32
  int halo;                    // 1: halo mode
  int box[3];                  // TMA box extent along w, h, d (elements, before element strides)
  int pw, plane_rows, plane_bytes;  // halo plane: row pitch, rows, bytes per half (1024-aligned)
  int sa, sb, tb;              // halo-mode ring depths (A planes, B stages) and taps per B stage
  int zs;                      // 1: z-streaming mode on raw lazy segments (sb = 0: resident weights)
  unsigned long long* range_events;  // fp16-pair range counter (z-streaming mode's in-kernel preparation)
};

struct OperandMaps {
  CUtensorMap seg[2];
};

template <int BC, int OP>
struct Cfg {
  static constexpr bool kSplit = OP == kOperandF16x2 || OP == kOperandTf32x2;
  static constexpr int kHalves = OP == kOperandTf32x2 ? 2 : 1;  // A boxes (128-byte rows) per K-step
  static constexpr int N = kSplit ? 2 * BC : BC;                // accumulator columns: stacked [W_hi; W_lo] rows
  static constexpr int kBRow = half_rows(OP) ? 64 : 128;        // bytes of one B row (32 channels)
  static constexpr int kAccBufs = (2 * N <= kTmemCols) ? 2 : 1;
  // epilogue warpgroups: with two accumulators each group drains every other tile (one warp per SM
  // sub-partition alone is latency-bound on the epilogue's dependent chains)
  static constexpr int kEpiGroups = kAccBufs;
  static constexpr int kThreadsC = 64 + 128 * kEpiGroups;
  static constexpr int kABytes = kHalves * BM * 128;
  static constexpr int kBBytes = N * kBRow;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kS0 = kStageBudget / kStageBytes;
  static constexpr int S = kS0 > 8 ? 8 : kS0;
  static_assert(S >= 2, "too few pipeline stages");
  static_assert(N % 16 == 0 && N <= 256, "MMA N");
};

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            int c4, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5, "
      "%6}], [%7];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// B-tile descriptor of the operand format (64-byte rows for the fp16 pair).
template <int OP>
__device__ __forceinline__ uint64_t b_desc_at(uint32_t saddr) {
  if constexpr (half_rows(OP)) return sw64_desc(saddr);
  else return sw128_desc(saddr);
}

// The MMAs of one K-step (32 input channels) into accumulator d.  ad: A rows
// (hi part), bd: B tile, lo16: offset of the TF32 lo rows (kOperandTf32x2),
// acc: 0 for the first K-step of a tile.  Descriptor offsets are in 16-byte
// units: the fp16 lo half of an A row starts 64 bytes in.
template <int BC, int OP>
__device__ __forceinline__ void kstep_mmas(uint32_t d, uint64_t ad, uint64_t bd, uint32_t lo16, uint32_t acc) {
  if constexpr (OP == kOperandF16x2) {
    constexpr uint32_t id2 = idesc_f16(BM, 2 * BC), id1 = idesc_f16(BM, BC);
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      mma_f16_ss(d, ad + 2 * kk, bd + 2 * kk, id2, (acc | kk) ? 1u : 0u);
      mma_f16_ss(d + BC, ad + 4 + 2 * kk, bd + 2 * kk, id1, 1u);
    }
  } else if constexpr (OP == kOperandBf16) {
    constexpr uint32_t id = idesc_bf16(BM, BC);
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) mma_f16_ss(d, ad + 2 * kk, bd + 2 * kk, id, (acc | kk) ? 1u : 0u);
  } else {
    constexpr uint32_t id = idesc_tf32(BM, Cfg<BC, OP>::N);
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      mma_tf32_ss(d, ad + 2 * kk, bd + 2 * kk, id, (acc | kk) ? 1u : 0u);
      if constexpr (OP == kOperandTf32x2) mma_tf32_ss(d, ad + lo16 + 2 * kk, bd + 2 * kk, id, 1u);
    }
  }
}

struct TileOrigin {
  int b, nt, t, d0, h0, w0;
};

__device__ __forceinline__ TileOrigin tile_origin(const Geometry& g, int tile) {
  TileOrigin o;
  o.nt = tile % g.n_tiles;
  const int mt = tile / g.n_tiles;
  o.b = mt / g.tps;
  o.t = mt - o.b * g.tps;
  const int plane = g.nh * g.nw;
  const int tdi = o.t / plane;
  const int rem = o.t - tdi * plane;
  const int thi = rem / g.nw;
  o.d0 = tdi * g.td;
  o.h0 = thi * g.th;
  o.w0 = (rem - thi * g.nw) * g.tw;
  return o;
}

// Channel chunk -> (tensor map, element coordinate of the hi box, of the lo box) for the two segments.
struct ChunkSource {
  const CUtensorMap* map;
  int c_hi, c_lo;
};

template <int OP>
__device__ __forceinline__ ChunkSource chunk_source(const nnb_conv3d_args& a, const Geometry& g,
                                                    const OperandMaps& maps, int chunk) {
  const int cg = chunk * BK;
  const bool second = cg >= g.c0len;
  const int cl = second ? cg - g.c0len : cg;
  const int cs = second ? a.seg[1].channels : g.c0len;
  if constexpr (half_rows(OP)) return ChunkSource{&maps.seg[second ? 1 : 0], 2 * cl, 0};  // [hi | lo] halves
  else return ChunkSource{&maps.seg[second ? 1 : 0], cl, cs + cl};
}

struct SharedMisc {
  uint64_t* bars;
  uint32_t* tmem_slot;
  volatile int* abort_flag;
  volatile int* votes;   // [4] stop votes of the first epilogue group
  volatile int* votes2;  // [4] of the second epilogue group
};

__device__ __forceinline__ SharedMisc shared_misc(uint8_t* misc) {
  SharedMisc m;
  m.bars = reinterpret_cast<uint64_t*>(misc);
  m.tmem_slot = reinterpret_cast<uint32_t*>(misc + 8 * kMaxBars);
  m.abort_flag = reinterpret_cast<volatile int*>(m.tmem_slot + 1);
  m.votes = reinterpret_cast<volatile int*>(m.tmem_slot + 2);
  m.votes2 = reinterpret_cast<volatile int*>(misc + 1792);
  return m;
}

// Coalesced store of this warp's 32 rows of 32 floats (lane = row): the rows pass through the warp's 2 KB
// shared staging buffer 16 at a time (16-byte chunks XOR-swizzled by row % 8) and every store
// instruction then writes four whole 128-byte rows, instead of one 16-byte piece of 32 rows.  dst: this
// lane's row destination (16-byte aligned), or nullptr to skip the row.  All 32 lanes must call it.
// kStats: while the rows are staged, lane c also reads column c of each staged row and accumulates, over
// the rows whose bit is set in vmask, the deviations from `shift` (the value of row 0): s += d, s2 += d^2.
// kChunks: only the first kChunks 16-byte chunks of each row are staged and written (4: a bf16 operand row,
// whose second half no MMA reads).
template <bool kStats = false, int kChunks = 8>
__device__ __forceinline__ void store_rows_staged(float4* stg, int lane, const float (&v)[32], float* dst,
                                                  unsigned vmask = 0u, float* shift = nullptr, float* s = nullptr,
                                                  float* s2 = nullptr) {
  const unsigned long long d = reinterpret_cast<unsigned long long>(dst);
  const float* f = reinterpret_cast<const float*>(stg);
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    if ((lane >> 4) == half) {
      const int r = lane & 15;
#pragma unroll
      for (int j = 0; j < kChunks; ++j)
        stg[r * 8 + (j ^ (r & 7))] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = 4 * i + (lane >> 3);  // staged row, 0..15
      const int c = lane & 7;
      const unsigned long long rd = __shfl_sync(0xffffffffu, d, half * 16 + r);
      const float4 val = stg[r * 8 + (c ^ (r & 7))];
      if (rd != 0ull && c < kChunks) reinterpret_cast<float4*>(rd)[c] = val;
    }
    if constexpr (kStats) {
      // column `lane` of staged row r: word 4 ((lane / 4) ^ (r % 8)) + lane % 4 of the row (conflict-free)
      float acc = 0.f, acc2 = 0.f;
#pragma unroll
      for (int r = 0; r < 16; ++r) {
        const float x = f[r * 32 + ((((lane >> 2) ^ (r & 7))) << 2) + (lane & 3)];
        if (half == 0 && r == 0) *shift = x;
        const float dv = (vmask >> (half * 16 + r)) & 1u ? x - *shift : 0.f;
        acc += dv;
        acc2 = fmaf(dv, dv, acc2);
      }
      *s += acc;
      *s2 += acc2;
    }
    __syncwarp();
  }
}

// Brick coordinates of an epilogue thread's row (fixed for the whole kernel: decompose it once).
struct RowPos {
  int row, dz, dy, dx;
};

__device__ __forceinline__ RowPos row_pos(const Geometry& g, int q, int lane) {
  RowPos r;
  r.row = q * 32 + lane;
  r.dz = r.row / (g.tw * g.th);
  r.dy = (r.row / g.tw) % g.th;
  r.dx = r.row % g.tw;
  return r;
}

// One finished accumulator -> outputs + partials (or the transposed-conv scatter).
// acc: TMEM address of the tile's (hi) accumulator columns for this warp's lanes; acc_lo: of the second
// accumulator of the split formats, or 0 when one accumulator holds every product (z-streaming mode).
// bar: named barrier of the four epilogue warps working on this tile; stg: this warp's staging buffer.
// stg_group: the staging buffers of the four warps of this epilogue group (2 KB each, in group order);
// widx: this warp's index in the group (the buffer it stages rows in).
template <int BC, int OP>
__device__ __forceinline__ void epilogue_tile(const nnb_conv3d_args& a, const Geometry& g, const TileOrigin& o,
                                              const RowPos& rp, uint32_t acc, uint32_t acc_lo, int lane,
                                              const float* __restrict__ col_inv, float4* stg_group, int widx,
                                              int bar = 1) {
  float4* stg = stg_group + widx * (kStagingBytes / 16);
  const int z = o.d0 + rp.dz, y = o.h0 + rp.dy, x = o.w0 + rp.dx;
  const bool valid = rp.row < g.rows && z < g.OD && y < g.OH && x < g.OW;
  const int64_t ovox = (int64_t)g.OD * g.OH * g.OW;
  const int64_t m = ((int64_t)z * g.OH + y) * g.OW + x;
  const unsigned vmask = __ballot_sync(0xffffffffu, valid);  // this warp's rows inside the output
#pragma unroll 1
  for (int cc = 0; cc < BC / 32; ++cc) {
    const int nbase = o.nt * BC + cc * 32;
    if (nbase >= a.cout) break;  // uniform across the epilogue warps
    float v[32];
    tmem_ld32(acc + cc * 32, v);
    if constexpr (OP == kOperandF16x2) {
      // (sum a_hi W0 + sum (a_hi W1 + a_lo W0)) / s of the column; acc_lo == 0: one accumulator holds all
      if (acc_lo != 0u) {
        float u[32];
        tmem_ld32(acc_lo + cc * 32, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] += u[i];
      }
      const float4* ci = reinterpret_cast<const float4*>(col_inv + nbase);  // 16-byte aligned
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 c4 = __ldg(ci + i);
        v[4 * i] *= c4.x;
        v[4 * i + 1] *= c4.y;
        v[4 * i + 2] *= c4.z;
        v[4 * i + 3] *= c4.w;
      }
    } else if constexpr (OP == kOperandTf32x2) {
      float u[32];
      tmem_ld32(acc_lo + cc * 32, u);
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] += u[i];
    }
    if (g.up_cout > 0) {
      // scatter: GEMM column n = tap * up_cout + channel of input voxel (z, y, x)
      const int tap = nbase / g.up_cout;
      const int co0 = nbase - tap * g.up_cout;
      float* dst = nullptr;
      if (valid) {
        const int ux = tap % g.UKW, uy = (tap / g.UKW) % g.UKH, uz = tap / (g.UKW * g.UKH);
        const int64_t OH2 = (int64_t)g.OH * g.UKH, OW2 = (int64_t)g.OW * g.UKW;
        const int64_t OD2 = (int64_t)g.OD * g.UKD;
        dst = a.out + ((((int64_t)o.b * OD2 + z * g.UKD + uz) * OH2 + y * g.UKH + uy) * OW2 + x * g.UKW + ux) *
                          g.up_cout + co0;
      }
      if (a.bias != nullptr) {
        const float4* b4 = reinterpret_cast<const float4*>(a.bias + co0);  // 16-byte aligned (checked on launch)
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 c4 = __ldg(b4 + i);
          v[4 * i] += c4.x;
          v[4 * i + 1] += c4.y;
          v[4 * i + 2] += c4.z;
          v[4 * i + 3] += c4.w;
        }
      }
      if (g.up_operand) {
        // the row's operand for the next convolution, 128 bytes at the same address as its 32 float32 values
        float pk[32];
        if constexpr (OP == kOperandF16x2) {
          // [hi(32) | lo(32)] fp16 (hi: 13 low mantissa bits cleared, lo = v - hi)
          bool over = false;
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float h0 = __uint_as_float(__float_as_uint(v[i]) & 0xFFFFE000u);
            const float h1 = __uint_as_float(__float_as_uint(v[i + 1]) & 0xFFFFE000u);
            const __half2 hh = __floats2half2_rn(h0, h1), ll = __floats2half2_rn(v[i] - h0, v[i + 1] - h1);
            pk[i / 2] = __uint_as_float(*reinterpret_cast<const uint32_t*>(&hh));
            pk[16 + i / 2] = __uint_as_float(*reinterpret_cast<const uint32_t*>(&ll));
            over |= fabsf(v[i]) >= 65504.f || fabsf(v[i + 1]) >= 65504.f;
          }
          if (over && valid) atomicAdd(g.range_events, 1ull);
        } else if constexpr (OP == kOperandBf16) {
          // [bf16(32) | (32)]: only the first half, which the MMAs read, is written
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const __nv_bfloat162 bb = __floats2bfloat162_rn(v[i], v[i + 1]);
            pk[i / 2] = __uint_as_float(*reinterpret_cast<const uint32_t*>(&bb));
            pk[16 + i / 2] = 0.f;
          }
        } else {
          // 32 TF32 values (round to nearest)
#pragma unroll
          for (int i = 0; i < 32; ++i) pk[i] = __uint_as_float(to_tf32(v[i]));
        }
        if constexpr (OP == kOperandBf16) store_rows_staged<false, 4>(stg, lane, pk, dst);
        else store_rows_staged(stg, lane, pk, dst);
      } else {
        store_rows_staged(stg, lane, v, dst);
      }
      continue;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (a.bias != nullptr && nbase + i < a.cout) v[i] += __ldg(a.bias + nbase + i);
      if (!valid) v[i] = 0.f;
    }
    const bool stats = a.partials != nullptr;  // uniform
    float shift = 0.f, cs = 0.f, cs2 = 0.f;
    if (nbase + 32 <= a.cout && (a.cout & 3) == 0) {  // uniform across the warp
      float* dst = valid ? a.out + ((int64_t)o.b * ovox + m) * a.cout + nbase : nullptr;
      if (stats) store_rows_staged<true>(stg, lane, v, dst, vmask, &shift, &cs, &cs2);
      else store_rows_staged(stg, lane, v, dst);
    } else {
      if (valid) {
        float* dst = a.out + ((int64_t)o.b * ovox + m) * a.cout + nbase;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (nbase + i < a.cout) dst[i] = v[i];
      }
      if (stats) store_rows_staged<true>(stg, lane, v, nullptr, vmask, &shift, &cs, &cs2);  // statistics only
    }
    if (stats) {
      // per-tile (sum, M2, n) of each column over the brick's valid rows: each warp's shifted sums give its
      // (sum, M2 around its mean, n); the group's first warp combines the four exactly (Chan et al.)
      const float nw = (float)__popc(vmask);
      const float sw = fmaf(nw, shift, cs);
      const float mw = nw > 0.f ? fmaf(-cs, cs / nw, cs2) : 0.f;
      float* mine = reinterpret_cast<float*>(stg);  // free: the warp's stores have read it
      mine[lane] = sw;
      mine[32 + lane] = fmaxf(mw, 0.f);
      if (lane == 0) mine[64] = nw;
      asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
      if (widx == 0 && nbase + lane < a.cout) {
        float sum = 0.f, n = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float* b = reinterpret_cast<const float*>(stg_group + w * (kStagingBytes / 16));
          sum += b[lane];
          n += b[64];
        }
        const float mean = n > 0.f ? sum / n : 0.f;
        float m2 = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float* b = reinterpret_cast<const float*>(stg_group + w * (kStagingBytes / 16));
          const float nb = b[64];
          if (nb > 0.f) {
            const float dm = b[lane] / nb - mean;
            m2 += fmaf(nb * dm, dm, b[32 + lane]);
          }
        }
        float* p = a.partials + (((int64_t)o.b * a.cout + nbase + lane) * g.tps + o.t) * 3;
        p[0] = sum;
        p[1] = m2;
        p[2] = n;
      }
      asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");  // the staging buffers are free again
    }
  }
}

// Epilogue warps' loop over this CTA's tiles (accumulator full/empty handshake).
template <int BC, int OP>
__device__ __forceinline__ void epilogue_role(const nnb_conv3d_args& a, const Geometry& g, int my_tiles,
                                              uint32_t tmem, const SharedMisc& sm, uint64_t* accf, uint64_t* acce,
                                              int warp, int lane, float4* stg_base) {
  using C = Cfg<BC, OP>;
  // fp16-pair images end with the per-column 1/s after the B tiles
  const float* col_inv = reinterpret_cast<const float*>(static_cast<const uint8_t*>(a.packed) +
                                                        (int64_t)g.n_tiles * g.ksteps * C::kBBytes);
  constexpr int NB = C::kAccBufs;
  const int q = warp & 3;  // warps 2..5 (and 6..9) own TMEM lane quarters 2, 3, 0, 1
  const int grp = C::kEpiGroups == 2 ? (warp - 2) >> 2 : 0;  // group grp drains accumulator grp
  const int bar = 1 + grp;
  volatile int* votes = grp ? sm.votes2 : sm.votes;
  const uint32_t lane_base = (uint32_t)(q * 32) << 16;
  const RowPos rp = row_pos(g, q, lane);
  for (int it = grp; it < my_tiles; it += C::kEpiGroups) {
    const int ab = NB == 2 ? (it & 1) : 0;
    const bool ok = mbar_wait(smem_u32(&accf[ab]), (it / NB) & 1, sm.abort_flag, 13);
    // consistent stop decision across the group's four warps
    if (lane == 0) votes[q] = (!ok || *sm.abort_flag) ? 1 : 0;
    asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
    const bool stop = votes[0] | votes[1] | votes[2] | votes[3];
    asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
    if (stop) break;
    fence_after();
    const TileOrigin o = tile_origin(g, blockIdx.x + it * gridDim.x);
    const uint32_t acc = tmem + ab * C::N + lane_base;
    epilogue_tile<BC, OP>(a, g, o, rp, acc, acc + BC, lane, col_inv, stg_base + 4 * grp * (kStagingBytes / 16),
                          (warp - 2) & 3, bar);
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&acce[ab]));
  }
}

__device__ __forceinline__ void tmem_alloc_all(uint32_t* slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(kTmemCols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_free_all(uint32_t tmem) {
  fence_after();
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// ---------------------------------------------------------------------------
// Box mode: one TMA box per half and one B tile per K-step (tap x 32 channels).
// ---------------------------------------------------------------------------
template <int BC, int OP>
__global__ void __launch_bounds__(Cfg<BC, OP>::kThreadsC, 1)
    conv3d_tc_kernel(const nnb_conv3d_args a, const Geometry g, const __grid_constant__ OperandMaps maps) {
  using C = Cfg<BC, OP>;
  constexpr int S = C::S;
  constexpr int NB = C::kAccBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;  // S x [A hi | A lo | B], each 1024-aligned
  const SharedMisc sm = shared_misc(smem + S * C::kStageBytes);
  int* kstab = reinterpret_cast<int*>(smem + S * C::kStageBytes + kMiscBytes);  // kx | ky<<4 | kz<<8 | chunk<<12
  float4* stg = reinterpret_cast<float4*>(smem + S * C::kStageBytes + kMiscBytes + 4 * kMaxKsteps);
  uint64_t* full = sm.bars;
  uint64_t* empty = sm.bars + S;
  uint64_t* accf = sm.bars + 2 * S;
  uint64_t* acce = sm.bars + 2 * S + 2;
  const uint32_t drain_bar = smem_u32(sm.bars + 2 * S + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int my_tiles = (g.total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(smem_u32(&full[s]), 1);   // producer's arrive.expect_tx, then the copies' bytes
      mbar_init(smem_u32(&empty[s]), 1);  // tcgen05.commit
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);  // accumulator full: tcgen05.commit
      mbar_init(smem_u32(&acce[i]), 4);  // accumulator empty: 4 epilogue warps
    }
    mbar_init(drain_bar, 1);
    *sm.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  const int taps = g.KD * g.KH * g.KW;
  for (int ks = threadIdx.x; ks < g.ksteps; ks += blockDim.x) {
    // chunk-major K order, the order of the weight image
    const int chunk = ks / taps, tap = ks - chunk * taps;
    const int kx = tap % g.KW, ky = (tap / g.KW) % g.KH, kz = tap / (g.KW * g.KH);
    kstab[ks] = kx | (ky << 4) | (kz << 8) | (chunk << 12);
  }
  if (warp == 1) tmem_alloc_all(sm.tmem_slot);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer -----------------------------
    if (lane == 0) {
      const uint32_t tx = (uint32_t)(C::kHalves * g.rows * 128 + C::kBBytes);
      int issued = 0;
      bool alive = true;
      for (int it = 0; it < my_tiles && alive; ++it) {
        const TileOrigin o = tile_origin(g, blockIdx.x + it * gridDim.x);
        const int wb = o.w0 * g.SW - g.PW, hb = o.h0 * g.SH - g.PH, db = o.d0 * g.SD - g.PD;
        const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(a.packed) + (int64_t)o.nt * g.ksteps * C::kBBytes;
        for (int ks = 0; ks < g.ksteps; ++ks) {
          const int G = it * g.ksteps + ks;
          const int s = G % S;
          if (G >= S && !mbar_wait(smem_u32(&empty[s]), ((G / S) - 1) & 1, sm.abort_flag, 12)) {
            alive = false;
            break;
          }
          const int e = kstab[ks];
          const ChunkSource src = chunk_source<OP>(a, g, maps, e >> 12);
          const int w = wb + (e & 15), h = hb + ((e >> 4) & 15), d = db + ((e >> 8) & 15);
          const uint32_t fb = smem_u32(&full[s]);
          const uint32_t st = smem_u32(stages + s * C::kStageBytes);
          mbar_arrive_expect_tx(fb, tx);
          tma_load_5d(st, src.map, src.c_hi, w, h, d, o.b, fb);
          if constexpr (C::kHalves == 2) tma_load_5d(st + BM * 128, src.map, src.c_lo, w, h, d, o.b, fb);
          bulk_g2s(st + C::kABytes, bsrc + (int64_t)ks * C::kBBytes, C::kBBytes, fb);
          issued = G + 1;
        }
      }
      if (*sm.abort_flag) {
        // wait (bounded) for the copies still in flight: the last S issued steps
        for (int G = std::max(0, issued - S); G < issued; ++G)
          mbar_wait(smem_u32(&full[G % S]), (G / S) & 1, sm.abort_flag, 15, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -------------------------------
    if (lane == 0) {
      // Descriptors are stage-0 bases plus constant offsets (start address in 16-byte units), so the
      // 4-8 MMAs of a K-step issue back to back with only adds between them.
      const uint64_t desc0 = sw128_desc(smem_u32(stages));
      const uint64_t bdesc0 = b_desc_at<OP>(smem_u32(stages) + C::kABytes);
      constexpr uint32_t kLo = (BM * 128) >> 4, kStage = C::kStageBytes >> 4;
      bool alive = true;
      int s = 0;
      uint32_t phase = 0;
      for (int it = 0; it < my_tiles && alive; ++it) {
        const int ab = NB == 2 ? (it & 1) : 0;
        if (it >= NB) {
          if (!mbar_wait(smem_u32(&acce[ab]), ((it / NB) - 1) & 1, sm.abort_flag, 14)) break;
          fence_after();
        }
        const uint32_t d = tmem + ab * C::N;
        for (int ks = 0; ks < g.ksteps; ++ks) {
          const uint64_t ad = desc0 + (uint64_t)(s * kStage);
          const uint64_t bd = bdesc0 + (uint64_t)(s * kStage);
          if (!mbar_wait(smem_u32(&full[s]), phase, sm.abort_flag, 11)) {
            alive = false;
            break;
          }
          fence_after();
          kstep_mmas<BC, OP>(d, ad, bd, kLo, ks > 0 ? 1u : 0u);
          mma_commit(smem_u32(&empty[s]));
          if (++s == S) {
            s = 0;
            phase ^= 1u;
          }
        }
        if (alive) mma_commit(smem_u32(&accf[ab]));
      }
      if (*sm.abort_flag) {
        // wait (bounded) for every MMA this thread issued before TMEM is freed
        mma_commit(drain_bar);
        mbar_wait(drain_bar, 0, sm.abort_flag, 16, false);
      }
    }
    __syncwarp();
  } else {
    epilogue_role<BC, OP>(a, g, my_tiles, tmem, sm, accf, acce, warp, lane, stg);
  }
  __syncthreads();
  if (warp == 1) tmem_free_all(tmem);
}

// ---------------------------------------------------------------------------
// Halo mode: one TMA box per (chunk, kz plane, half) feeds every (kx, ky) tap.
// ---------------------------------------------------------------------------
// TB = taps per B stage: 3 (a whole kx row of a 3-wide kernel, fully unrolled) or 1 (any kernel).
template <int BC, int OP, int TB>
__global__ void __launch_bounds__(Cfg<BC, OP>::kThreadsC, 1)
    conv3d_halo_kernel(const nnb_conv3d_args a, const Geometry g, const __grid_constant__ OperandMaps maps) {
  using C = Cfg<BC, OP>;
  constexpr int NB = C::kAccBufs;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int SA = g.sa, SB = g.sb;
  const int a_stage = C::kHalves * g.plane_bytes;
  const uint32_t b_stage = (uint32_t)(g.tb * C::kBBytes);
  const int taps = g.KD * g.KH * g.KW;
  uint8_t* a_ring = smem;                    // SA x [plane hi | plane lo], 1024-aligned
  uint8_t* b_ring = smem + SA * a_stage;     // SB x tb B tiles, 1024-aligned
  const SharedMisc sm = shared_misc(b_ring + SB * b_stage);
  uint64_t* a_full = sm.bars;
  uint64_t* a_empty = sm.bars + SA;
  uint64_t* b_full = sm.bars + 2 * SA;
  uint64_t* b_empty = sm.bars + 2 * SA + SB;
  uint64_t* accf = sm.bars + 2 * SA + 2 * SB;
  uint64_t* acce = accf + 2;
  const uint32_t drain_bar = smem_u32(accf + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int my_tiles = (g.total_tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  const int taps2d = g.KH * g.KW;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(smem_u32(&a_full[s]), 1);
      mbar_init(smem_u32(&a_empty[s]), 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(smem_u32(&b_full[s]), 1);
      mbar_init(smem_u32(&b_empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), 4);
    }
    mbar_init(drain_bar, 1);
    *sm.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc_all(sm.tmem_slot);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    // ------------------------------ TMA producer -----------------------------
    if (lane == 0) {
      const uint32_t tx_a = (uint32_t)(C::kHalves * g.plane_rows * 128);
      int P = 0, T = 0;
      bool alive = true;
      for (int it = 0; it < my_tiles && alive; ++it) {
        const TileOrigin o = tile_origin(g, blockIdx.x + it * gridDim.x);
        const int wb = o.w0 - g.PW, hb = o.h0 - g.PH, db = o.d0 - g.PD;
        const uint8_t* bsrc = reinterpret_cast<const uint8_t*>(a.packed) + (int64_t)o.nt * g.ksteps * C::kBBytes;
        for (int c = 0; c < g.nchunk && alive; ++c) {
          const ChunkSource src = chunk_source<OP>(a, g, maps, c);
          for (int kz = 0; kz < g.KD && alive; ++kz) {
            const int sa = P % SA;
            if (P >= SA && !mbar_wait(smem_u32(&a_empty[sa]), ((P / SA) - 1) & 1, sm.abort_flag, 22)) {
              alive = false;
              break;
            }
            const uint32_t fa = smem_u32(&a_full[sa]);
            const uint32_t dst = smem_u32(a_ring + sa * a_stage);
            mbar_arrive_expect_tx(fa, tx_a);
            tma_load_5d(dst, src.map, src.c_hi, wb, hb, db + kz, o.b, fa);
            if constexpr (C::kHalves == 2)
              tma_load_5d(dst + g.plane_bytes, src.map, src.c_lo, wb, hb, db + kz, o.b, fa);
            ++P;
            for (int t2 = 0; t2 < taps2d; t2 += g.tb) {
              const int sb = T % SB;
              if (T >= SB && !mbar_wait(smem_u32(&b_empty[sb]), ((T / SB) - 1) & 1, sm.abort_flag, 23)) {
                alive = false;
                break;
              }
              // tb consecutive taps of one (chunk, kz, ky) row: contiguous in the chunk-major image
              const int tap = kz * taps2d + t2;
              const uint32_t fb = smem_u32(&b_full[sb]);
              mbar_arrive_expect_tx(fb, b_stage);
              bulk_g2s(smem_u32(b_ring + sb * b_stage), bsrc + (int64_t)(c * taps + tap) * C::kBBytes, b_stage, fb);
              ++T;
            }
          }
        }
      }
      if (*sm.abort_flag) {
        for (int i = std::max(0, P - SA); i < P; ++i)
          mbar_wait(smem_u32(&a_full[i % SA]), (i / SA) & 1, sm.abort_flag, 25, false);
        for (int i = std::max(0, T - SB); i < T; ++i)
          mbar_wait(smem_u32(&b_full[i % SB]), (i / SB) & 1, sm.abort_flag, 26, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -------------------------------
    if (lane == 0) {
      // Stage-0 descriptor bases plus constant offsets (16-byte units): A planes with 8-row groups
      // pw rows apart, B tiles with the format's usual groups.
      const uint64_t adesc0 = sw128_desc(smem_u32(a_ring), (uint32_t)g.pw * 128);
      const uint64_t bdesc0 = b_desc_at<OP>(smem_u32(b_ring));
      const uint32_t a_stage16 = (uint32_t)a_stage >> 4, lo16 = (uint32_t)g.plane_bytes >> 4;
      const uint32_t b_stage16 = b_stage >> 4;
      constexpr uint32_t kB16 = C::kBBytes >> 4;
      int sa = 0, sb = 0;
      uint32_t pa = 0, pb = 0;
      bool alive = true;
      for (int it = 0; it < my_tiles && alive; ++it) {
        const int ab = NB == 2 ? (it & 1) : 0;
        if (it >= NB) {
          if (!mbar_wait(smem_u32(&acce[ab]), ((it / NB) - 1) & 1, sm.abort_flag, 24)) break;
          fence_after();
        }
        const uint32_t d = tmem + ab * C::N;
        uint32_t accumulate = 0;
        for (int c = 0; c < g.nchunk && alive; ++c) {
          for (int kz = 0; kz < g.KD && alive; ++kz) {
            const uint64_t ap = adesc0 + (uint64_t)(sa * a_stage16);
            if (!mbar_wait(smem_u32(&a_full[sa]), pa, sm.abort_flag, 21)) {
              alive = false;
              break;
            }
            fence_after();
            if constexpr (TB > 1) {
              // one B stage per kx row (TB == KW): compile-time tap offsets, no control flow between
              // the row's 8 x TB MMAs
              for (int ky = 0; ky < g.KH && alive; ++ky) {
                const uint64_t arow = ap + (uint64_t)(ky * g.pw * 8);
                const uint64_t bstage_desc = bdesc0 + (uint64_t)(sb * b_stage16);
                if (!mbar_wait(smem_u32(&b_full[sb]), pb, sm.abort_flag, 27)) {
                  alive = false;
                  break;
                }
                fence_after();
#pragma unroll
                for (int j = 0; j < TB; ++j)
                  kstep_mmas<BC, OP>(d, arow + (uint64_t)(8 * j), bstage_desc + (uint64_t)(j * kB16), lo16,
                                     accumulate | (uint32_t)j);
                accumulate = 1;
                mma_commit(smem_u32(&b_empty[sb]));
                if (++sb == SB) {
                  sb = 0;
                  pb ^= 1u;
                }
              }
            } else {
            // A row offset of tap (kx, ky) in 16-byte units, advanced incrementally (no divisions
            // between MMA groups): +8 per kx, +8 * (pw - KW + 1) at the end of a kx row.
            uint32_t aoff = 0;
            int kx = 0;
            const uint32_t row_wrap = (uint32_t)(g.pw - g.KW + 1) * 8;
            for (int t2 = 0; t2 < taps2d && alive; t2 += g.tb) {
              const uint64_t bstage_desc = bdesc0 + (uint64_t)(sb * b_stage16);
              if (!mbar_wait(smem_u32(&b_full[sb]), pb, sm.abort_flag, 27)) {
                alive = false;
                break;
              }
              fence_after();
              uint64_t bd = bstage_desc;
              for (int j = 0; j < g.tb; ++j) {
                const uint64_t ad = ap + aoff;
                if (++kx == g.KW) {
                  kx = 0;
                  aoff += row_wrap;
                } else {
                  aoff += 8;
                }
                kstep_mmas<BC, OP>(d, ad, bd, lo16, accumulate);
                accumulate = 1;
                bd += kB16;
              }
              mma_commit(smem_u32(&b_empty[sb]));
              if (++sb == SB) {
                sb = 0;
                pb ^= 1u;
              }
            }
            }
            mma_commit(smem_u32(&a_empty[sa]));
            if (++sa == SA) {
              sa = 0;
              pa ^= 1u;
            }
          }
        }
        if (alive) mma_commit(smem_u32(&accf[ab]));
      }
      if (*sm.abort_flag) {
        mma_commit(drain_bar);
        mbar_wait(drain_bar, 0, sm.abort_flag, 16, false);
      }
    }
    __syncwarp();
  } else {
    epilogue_role<BC, OP>(a, g, my_tiles, tmem, sm, accf, acce, warp, lane,
                          reinterpret_cast<float4*>(b_ring + SB * b_stage + kMiscBytes));
  }
  __syncthreads();
  if (warp == 1) tmem_free_all(tmem);
}

// ---------------------------------------------------------------------------
// Z-streaming mode (3x3x3, stride 1, padding 1, <= 32 output channels; fp16
// pairs, and the single-product bf16 and TF32 formats).  The 128^3 stages' layers: a CTA walks a contiguous run of the
// output planes of 8 (w) x 16 (h) brick columns (column-major, z fastest; the
// runs of all CTAs split the volume's planes evenly).  Each input plane u of a
// column is loaded once (one halo plane box per 32-channel chunk) and, per
// (ky, kx) tap and 16-channel sub-step, multiplied by the weights of all
// three kz taps stacked along N (N = 96; block kz feeds output plane
// u + 1 - kz), three products into the same accumulators:
//   A_hi x [W0(kz0); W0(kz1); W0(kz2)],  A_hi x [W1(kz0..2)],  A_lo x [W0(kz0..2)].
// The accumulators of consecutive output planes sit in a TMEM ring of 16
// slots of 32 columns, slot 15 - (P mod 16) for the P-th plane of the CTA's
// sequence, so the three planes an input feeds occupy adjacent ascending
// slots and one MMA covers them (two where the ring wraps, 1 plane in 8).
// Output plane u - 1 is complete after input u.  The epilogue reads a
// complete plane, writes it (planes outside the run -- the halo planes of a
// partial column -- are only discarded), zeroes its slot and releases it, so
// every MMA accumulates.  A column costs 3 MMAs per (tap, sub-step, input
// plane) instead of 6 per output plane, and each input plane is read once
// instead of three times.  The single-product formats stack only [W(kz0..2)]
// (96 rows) and issue one MMA per (tap, sub-step): bf16 sub-steps of 16
// channels, TF32 sub-steps of 8 channels with 128-byte B rows.  The input planes are the raw float32 activation
// (a lazy segment of the previous layer): two transform warps convert each
// landed plane in place -- instance-norm affine + LeakyReLU, zero for the
// padding rows, fp16 hi / lo split into the MMA's [hi | lo] row layout and
// the fp16 range count (bf16: the hi half only; TF32: the row rounded to
// TF32 in place) -- so the activation makes no extra trip through HBM.  The 27 taps' weights of a single-chunk layer stay
// resident in shared memory for the whole kernel (rearranged from the weight
// image by bulk copies); wider inputs stream one (chunk, ky) row of stacked
// weights per stage.
// ---------------------------------------------------------------------------
constexpr int kZsSlots = 16;

// Stacked B rows per (ky, kx) tap: fp16 pairs [W0 x 3 kz ; W1 x 3 kz], the single formats [W x 3 kz].
__host__ __device__ constexpr int zs_rows(int op) { return op == kOperandF16x2 ? 6 * 32 : 3 * 32; }
__host__ __device__ constexpr int zs_row_bytes(int op) { return half_rows(op) ? 64 : 128; }
__host__ __device__ constexpr int zs_tap_bytes(int op) { return zs_rows(op) * zs_row_bytes(op); }

// The work split (zs_schedule.cuh) over this launch's geometry.
__host__ __device__ __forceinline__ ZsRun zs_run(const Geometry& g, int cta, int ncta) {
  return zs_run((int64_t)g.total_tiles, g.OD, cta, ncta);  // total_tiles = brick columns x OD
}

__host__ __device__ __forceinline__ bool zs_next(const Geometry& g, ZsRun& r, ZsSegment& s, int cta, int ncta) {
  return zs_next(r, s, g.OD, g.ID, cta, ncta);
}

__device__ __forceinline__ int zs_slot(int P) { return kZsSlots - 1 - (P & (kZsSlots - 1)); }

// The MMAs of one row of taps (ky fixed; kx = 0..2; 16-channel sub-steps, or 8-channel ones for TF32) into the
// slots of the three planes an input feeds (d: TMEM address of slot s0).  N1 = 3: the slots s0..s0+2 are adjacent,
// one MMA of N = 96 per product; N1 = 1 or 2: the ring wraps after N1 blocks, so each MMA splits into N = 32 N1
// at s0 and N = 32 (3 - N1) at slot 0.  arow / brow: A (hi) and stacked-B descriptors of the row's kx = 0 tap;
// the lo half of an fp16-pair A row starts 64 bytes in, the W1 blocks 96 B rows in.
template <int OP, int N1>
__device__ __forceinline__ void zs_row(uint32_t tmem, uint32_t d, uint64_t arow, uint64_t brow) {
  constexpr uint32_t kTap16 = (uint32_t)zs_tap_bytes(OP) >> 4;
  constexpr uint32_t kBlk16 = (uint32_t)(32 * zs_row_bytes(OP)) >> 4;  // one kz block of 32 B rows
  constexpr uint32_t kSplit16 = N1 * kBlk16;
  if constexpr (OP == kOperandF16x2) {
    constexpr uint32_t kW116 = 3 * kBlk16;
    constexpr uint32_t idA = idesc_f16(BM, 32 * N1);
#pragma unroll
    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint64_t ad = arow + (uint64_t)(8 * kx + 2 * kk);
        const uint64_t bd = brow + (uint64_t)(kx * kTap16 + 2 * kk);
        mma_f16_ss(d, ad, bd, idA, 1u);
        mma_f16_ss(d, ad, bd + kW116, idA, 1u);
        mma_f16_ss(d, ad + 4, bd, idA, 1u);
        if constexpr (N1 < 3) {
          constexpr uint32_t idB = idesc_f16(BM, 32 * (3 - N1));
          mma_f16_ss(tmem, ad, bd + kSplit16, idB, 1u);
          mma_f16_ss(tmem, ad, bd + kW116 + kSplit16, idB, 1u);
          mma_f16_ss(tmem, ad + 4, bd + kSplit16, idB, 1u);
        }
      }
  } else if constexpr (OP == kOperandBf16) {
    constexpr uint32_t idA = idesc_bf16(BM, 32 * N1);
#pragma unroll
    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const uint64_t ad = arow + (uint64_t)(8 * kx + 2 * kk);
        const uint64_t bd = brow + (uint64_t)(kx * kTap16 + 2 * kk);
        mma_f16_ss(d, ad, bd, idA, 1u);
        if constexpr (N1 < 3) mma_f16_ss(tmem, ad, bd + kSplit16, idesc_bf16(BM, 32 * (3 - N1)), 1u);
      }
  } else {
    static_assert(OP == kOperandTf32, "z-streaming formats: fp16 pair, bf16, TF32");
    constexpr uint32_t idA = idesc_tf32(BM, 32 * N1);
#pragma unroll
    for (int kx = 0; kx < 3; ++kx)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t ad = arow + (uint64_t)(8 * kx + 2 * kk);
        const uint64_t bd = brow + (uint64_t)(kx * kTap16 + 2 * kk);
        mma_tf32_ss(d, ad, bd, idA, 1u);
        if constexpr (N1 < 3) mma_tf32_ss(tmem, ad, bd + kSplit16, idesc_tf32(BM, 32 * (3 - N1)), 1u);
      }
  }
}

// producer, MMA issuer, two epilogue warpgroups taking alternate planes, two operand-transform warps
constexpr int kZsThreads = 12 * 32;

// In-place conversion of one landed raw plane box (rows of 32 float32 channels, 128-byte swizzled) into the
// rows the MMA reads, by 64 threads, one whole row per thread at a time (the row's eight 16-byte chunks are
// all read before any is written, so no other thread touches it): fp16 pairs [hi(32) | lo(32)], bf16 the hi
// half only, TF32 the 32 values rounded to TF32 in place.  aff: the chunk's 32 scales then 32 shifts
// (identity for a raw segment).  Padding rows become zeros.  Returns whether any value reached the fp16
// range limit (fp16 pairs only).
template <int OP>
__device__ __forceinline__ bool zs_transform_plane(uint8_t* plane, const Geometry& g, const float* aff,
                                                   bool leaky_act, int w0, int h0, float slope, int t) {
  float amax = 0.f;
  // the chunk's affine in registers for the whole plane (not re-read from shared memory per row), as channel
  // pairs for packed f32x2 arithmetic (each half is the scalar operation with the same rounding)
  unsigned long long sc2[16], sh2[16], slope2;
#pragma unroll
  for (int k = 0; k < 16; ++k) {
    sc2[k] = *reinterpret_cast<const unsigned long long*>(aff + 2 * k);
    sh2[k] = *reinterpret_cast<const unsigned long long*>(aff + 32 + 2 * k);
  }
  asm("mov.b64 %0, {%1, %1};" : "=l"(slope2) : "f"(slope));
  for (int r = t; r < g.plane_rows; r += 64) {
    uint8_t* row = plane + r * 128;
    const int sw = r & 7;
    const int hh = r / g.pw, ww = r - hh * g.pw;
    if ((unsigned)(w0 + ww) >= (unsigned)g.IW || (unsigned)(h0 + hh) >= (unsigned)g.IH) {
      // padding row: the normalised activation there is zero
#pragma unroll
      for (int k = 0; k < 8; ++k) *reinterpret_cast<uint4*>(row + (k << 4)) = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    float4 x[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) x[k] = *reinterpret_cast<const float4*>(row + ((k ^ sw) << 4));
    uint32_t hi[16], lo[16];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float v[4];
      {
        unsigned long long x01, x23, y01, y23;
        asm("mov.b64 %0, {%1, %2};" : "=l"(x01) : "f"(x[k].x), "f"(x[k].y));
        asm("mov.b64 %0, {%1, %2};" : "=l"(x23) : "f"(x[k].z), "f"(x[k].w));
        asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(y01) : "l"(x01), "l"(sc2[2 * k]), "l"(sh2[2 * k]));
        asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(y23) : "l"(x23), "l"(sc2[2 * k + 1]), "l"(sh2[2 * k + 1]));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(v[0]), "=f"(v[1]) : "l"(y01));
        asm("mov.b64 {%0, %1}, %2;" : "=f"(v[2]), "=f"(v[3]) : "l"(y23));
        if (leaky_act) {
          // LeakyReLU for 0 <= slope <= 1: max(v, v * slope)
          unsigned long long m01, m23;
          float m[4];
          asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(m01) : "l"(y01), "l"(slope2));
          asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(m23) : "l"(y23), "l"(slope2));
          asm("mov.b64 {%0, %1}, %2;" : "=f"(m[0]), "=f"(m[1]) : "l"(m01));
          asm("mov.b64 {%0, %1}, %2;" : "=f"(m[2]), "=f"(m[3]) : "l"(m23));
#pragma unroll
          for (int e = 0; e < 4; ++e) v[e] = fmaxf(v[e], m[e]);
        }
      }
      if constexpr (OP == kOperandF16x2) {
        float h[4], l[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          amax = fmaxf(amax, fabsf(v[e]));
          // hi: v with the 13 low mantissa bits cleared (exactly an fp16 value in fp16's normal range),
          // lo = v - hi exactly; both are then rounded to fp16
          h[e] = __uint_as_float(__float_as_uint(v[e]) & 0xFFFFE000u);
          l[e] = v[e] - h[e];
        }
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const __half2 hh2 = __floats2half2_rn(h[e], h[e + 1]);
          const __half2 ll2 = __floats2half2_rn(l[e], l[e + 1]);
          hi[2 * k + e / 2] = *reinterpret_cast<const uint32_t*>(&hh2);
          lo[2 * k + e / 2] = *reinterpret_cast<const uint32_t*>(&ll2);
        }
      } else if constexpr (OP == kOperandBf16) {
#pragma unroll
        for (int e = 0; e < 4; e += 2) {
          const __nv_bfloat162 bb = __floats2bfloat162_rn(v[e], v[e + 1]);
          hi[2 * k + e / 2] = *reinterpret_cast<const uint32_t*>(&bb);
        }
      } else {
        // TF32: logical chunk k holds channels 4k..4k+3 as 32-bit values (every chunk was read above)
        *reinterpret_cast<uint4*>(row + ((k ^ sw) << 4)) = make_uint4(to_tf32(v[0]), to_tf32(v[1]), to_tf32(v[2]),
                                                                      to_tf32(v[3]));
      }
    }
    if constexpr (half_rows(OP)) {
      // hi halves of channels 8m..8m+7 form logical chunk m, the lo halves (fp16 pairs) chunk 4 + m
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        *reinterpret_cast<uint4*>(row + ((m ^ sw) << 4)) =
            make_uint4(hi[4 * m], hi[4 * m + 1], hi[4 * m + 2], hi[4 * m + 3]);
        if constexpr (OP == kOperandF16x2)
          *reinterpret_cast<uint4*>(row + (((4 + m) ^ sw) << 4)) =
              make_uint4(lo[4 * m], lo[4 * m + 1], lo[4 * m + 2], lo[4 * m + 3]);
      }
    }
  }
  return amax >= 65504.f;
}

// This warp's copy of the chunks' affine table for sample b (warp-local: no barrier another warp could miss).
__device__ __forceinline__ void zs_load_affine(const nnb_conv3d_args& a, const Geometry& g, int b, float* aff,
                                               int lane) {
  __syncwarp();  // the warp no longer reads the previous sample's table
  for (int i = lane; i < g.nchunk * 64; i += 32) {
    const int c = i >> 6, k = i & 63, ch = k & 31;
    const int cg = c * BK;
    const bool second = cg >= g.c0len;
    const nnb_segment& seg = a.seg[second ? 1 : 0];
    const int idx = b * seg.channels + (second ? cg - g.c0len : cg) + ch;
    float v = k < 32 ? 1.f : 0.f;
    if (seg.scale != nullptr) v = k < 32 ? __ldg(seg.scale + idx) : __ldg(seg.shift + idx);
    aff[i] = v;
  }
  __syncwarp();
}

template <int OP>
__global__ void __launch_bounds__(kZsThreads, 1)
    conv3d_zstream_kernel(const nnb_conv3d_args a, const Geometry g, const __grid_constant__ OperandMaps maps) {
  constexpr int BC = 32;
  using C = Cfg<BC, OP>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int SA = g.sa, SB = g.sb;
  const bool resident = SB == 0;
  const int a_entry = g.nchunk * g.plane_bytes;              // one input plane, all chunks
  constexpr uint32_t kTapBytes = zs_tap_bytes(OP);         // stacked weights of one (ky, kx) tap
  constexpr uint32_t kBlkBytes = 32 * zs_row_bytes(OP);     // one kz block (32 B rows) of a part
  constexpr int kParts = OP == kOperandF16x2 ? 2 : 1;       // [W0 ; W1] or [W] per image tile
  const uint32_t b_stage = 3u * kTapBytes;                  // one (chunk, ky) row of taps
  const uint32_t b_bytes = resident ? (uint32_t)g.nchunk * 9u * kTapBytes : (uint32_t)SB * b_stage;
  uint8_t* a_ring = smem;
  uint8_t* b_ring = smem + SA * a_entry;
  const SharedMisc sm = shared_misc(b_ring + b_bytes);
  uint64_t* a_full = sm.bars;         // raw plane landed (TMA)
  uint64_t* a_empty = a_full + SA;
  uint64_t* a_ready = a_empty + SA;   // plane converted to MMA operand rows (transform warps)
  uint64_t* b_full = a_ready + SA;    // SB stages, or [0] = resident weights
  uint64_t* b_empty = b_full + max(SB, 1);
  uint64_t* accf = b_empty + max(SB, 1);
  uint64_t* acce = accf + kZsSlots;
  const uint32_t drain_bar = smem_u32(acce + kZsSlots);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int bricks = g.nh * g.nw;
  // per transform warp: [nchunk][scale 32 | shift 32]
  float* aff = reinterpret_cast<float*>(b_ring + b_bytes + kMiscBytes) + (warp >= 10 ? (warp - 10) * g.nchunk * 64 : 0);
  // eight epilogue warps' staging buffers after the two affine tables
  float4* zs_stg = reinterpret_cast<float4*>(b_ring + b_bytes + kMiscBytes + 2 * g.nchunk * 64 * 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < SA; ++s) {
      mbar_init(smem_u32(&a_full[s]), 1);
      mbar_init(smem_u32(&a_empty[s]), 1);
      mbar_init(smem_u32(&a_ready[s]), 2);
    }
    for (int s = 0; s < max(SB, 1); ++s) {
      mbar_init(smem_u32(&b_full[s]), 1);
      mbar_init(smem_u32(&b_empty[s]), 1);
    }
    for (int i = 0; i < kZsSlots; ++i) {
      mbar_init(smem_u32(&accf[i]), 1);
      mbar_init(smem_u32(&acce[i]), 4);
    }
    mbar_init(drain_bar, 1);
    *sm.abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc_all(sm.tmem_slot);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *sm.tmem_slot;
  if (warp >= 2 && warp < 6) {
    // every slot starts at zero: the MMAs always accumulate
    const uint32_t lanes = (uint32_t)((warp & 3) * 32) << 16;
#pragma unroll 1
    for (int c = 0; c < kTmemCols; c += 32) tmem_zero32(tmem + lanes + (uint32_t)c);
  }
  fence_before();
  __syncthreads();
  fence_after();

  const uint8_t* wimg = static_cast<const uint8_t*>(a.packed);
  const int taps = 27;
  if (warp == 0) {
    // ------------------------------ TMA producer -----------------------------
    if (lane == 0) {
      bool alive = true;
      if (resident) {
        // per chunk, the stacked rows of tap (ky, kx): [W0(kz0..2) ; W1(kz0..2)] (or [W(kz0..2)]), 32 rows each,
        // from the image's [W0 ; W1] (or [W]) tile of K-step (chunk, tap (kz, ky, kx))
        const uint32_t fb = smem_u32(&b_full[0]);
        mbar_arrive_expect_tx(fb, (uint32_t)g.nchunk * 9u * kTapBytes);
        for (int c = 0; c < g.nchunk; ++c)
          for (int t = 0; t < 9; ++t)
            for (int part = 0; part < kParts; ++part)
              for (int kz = 0; kz < 3; ++kz)
                bulk_g2s(smem_u32(b_ring + (c * 9 + t) * kTapBytes + (part * 3 + kz) * kBlkBytes),
                         wimg + (int64_t)(c * taps + kz * 9 + t) * C::kBBytes + part * kBlkBytes, kBlkBytes, fb);
      }
      int P = 0, T = 0;
      ZsRun run = zs_run(g, (int)blockIdx.x, (int)gridDim.x);
      ZsSegment sg;
      while (alive && zs_next(g, run, sg, (int)blockIdx.x, (int)gridDim.x)) {
        const int b = sg.col / bricks, rem = sg.col - b * bricks;
        const int hb = rem / g.nw, wb = rem - hb * g.nw;
        const int w0 = wb * kHaloW - 1, h0 = hb * kHaloH - 1;
        for (int u = sg.ua; u <= sg.ub && alive; ++u) {
          const int sa = P % SA;
          if (P >= SA && !mbar_wait(smem_u32(&a_empty[sa]), ((P / SA) - 1) & 1, sm.abort_flag, 32)) {
            alive = false;
            break;
          }
          const uint32_t fa = smem_u32(&a_full[sa]);
          mbar_arrive_expect_tx(fa, (uint32_t)(g.nchunk * g.plane_rows * 128));
          for (int c = 0; c < g.nchunk; ++c) {
            // raw float32 plane of the chunk's 32 channels, or its operand rows when prepared
            const ChunkSource src = a.seg[c * BK >= g.c0len ? 1 : 0].prepared
                                        ? chunk_source<OP>(a, g, maps, c)
                                        : chunk_source<kOperandTf32>(a, g, maps, c);
            tma_load_5d(smem_u32(a_ring + sa * a_entry + c * g.plane_bytes), src.map, src.c_hi, w0, h0, u, b, fa);
          }
          ++P;
          if (!resident) {
            for (int c = 0; c < g.nchunk && alive; ++c)
              for (int ky = 0; ky < 3; ++ky) {
                const int sb = T % SB;
                if (T >= SB && !mbar_wait(smem_u32(&b_empty[sb]), ((T / SB) - 1) & 1, sm.abort_flag, 33)) {
                  alive = false;
                  break;
                }
                const uint32_t fb = smem_u32(&b_full[sb]);
                mbar_arrive_expect_tx(fb, b_stage);
                uint8_t* dst = b_ring + sb * b_stage;
                for (int kx = 0; kx < 3; ++kx)
                  for (int part = 0; part < kParts; ++part)
                    for (int kz = 0; kz < 3; ++kz)
                      bulk_g2s(smem_u32(dst + kx * kTapBytes + (part * 3 + kz) * kBlkBytes),
                               wimg + (int64_t)(c * taps + kz * 9 + ky * 3 + kx) * C::kBBytes + part * kBlkBytes,
                               kBlkBytes, fb);
                ++T;
              }
          }
        }
      }
      if (*sm.abort_flag) {
        for (int i = max(0, P - SA); i < P; ++i)
          mbar_wait(smem_u32(&a_full[i % SA]), (i / SA) & 1, sm.abort_flag, 34, false);
        if (resident) mbar_wait(smem_u32(&b_full[0]), 0, sm.abort_flag, 35, false);
        for (int i = max(0, T - SB); i < T; ++i)
          mbar_wait(smem_u32(&b_full[i % SB]), (i / SB) & 1, sm.abort_flag, 35, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer -------------------------------
    if (lane == 0) {
      const uint64_t adesc0 = sw128_desc(smem_u32(a_ring), (uint32_t)g.pw * 128);
      const uint64_t bdesc0 = b_desc_at<OP>(smem_u32(b_ring));
      const uint32_t entry16 = (uint32_t)a_entry >> 4, plane16 = (uint32_t)g.plane_bytes >> 4;
      const uint32_t row16 = (uint32_t)g.pw * 8;  // one ky step of the plane in 16-byte units
      constexpr uint32_t kTap16 = kTapBytes >> 4;
      const uint32_t stage16 = b_stage >> 4;
      bool alive = true;
      if (resident) alive = mbar_wait(smem_u32(&b_full[0]), 0, sm.abort_flag, 36);
      if (alive) fence_after();
      int P = 0, PA = 0, T = 0;
      int acquired = -1;  // planes [0, acquired] have had their slot released by its previous plane
      ZsRun run = zs_run(g, (int)blockIdx.x, (int)gridDim.x);
      ZsSegment sg;
      while (alive && zs_next(g, run, sg, (int)blockIdx.x, (int)gridDim.x)) {
        // planes ua - 1 .. ub + 1 of this segment are P .. P + (ub - ua) + 2
        for (int u = sg.ua; u <= sg.ub && alive; ++u) {
          const int Pn = P + (u - sg.ua) + 2;  // plane u + 1: this input's first contribution
          for (int p = acquired + 1; p <= Pn && alive; ++p)
            if (p >= kZsSlots && !mbar_wait(smem_u32(&acce[zs_slot(p)]), ((p / kZsSlots) - 1) & 1, sm.abort_flag, 37))
              alive = false;
          if (!alive) break;
          acquired = Pn;
          const int sa = PA % SA;
          if (!mbar_wait(smem_u32(&a_ready[sa]), (PA / SA) & 1, sm.abort_flag, 38)) {
            alive = false;
            break;
          }
          fence_after();
          const int s0 = zs_slot(Pn);
          const uint32_t dslot = tmem + 32u * (uint32_t)s0;
          for (int c = 0; c < g.nchunk && alive; ++c) {
            const uint64_t ap = adesc0 + (uint64_t)(sa * entry16 + c * plane16);
            if (resident) {
              const uint64_t bchunk = bdesc0 + (uint64_t)(c * 9) * kTap16;  // this chunk's resident taps
              // the wrap case is uniform per input plane: one straight-line row variant per case
              if (s0 <= kZsSlots - 3) {
#pragma unroll 1
                for (int ky = 0; ky < 3; ++ky)
                  zs_row<OP, 3>(tmem, dslot, ap + (uint64_t)(ky * row16), bchunk + (uint64_t)(ky * 3 * kTap16));
              } else if (s0 == kZsSlots - 2) {
#pragma unroll 1
                for (int ky = 0; ky < 3; ++ky)
                  zs_row<OP, 2>(tmem, dslot, ap + (uint64_t)(ky * row16), bchunk + (uint64_t)(ky * 3 * kTap16));
              } else {
#pragma unroll 1
                for (int ky = 0; ky < 3; ++ky)
                  zs_row<OP, 1>(tmem, dslot, ap + (uint64_t)(ky * row16), bchunk + (uint64_t)(ky * 3 * kTap16));
              }
            } else {
              for (int ky = 0; ky < 3; ++ky) {
                const int sb = T % SB;
                if (!mbar_wait(smem_u32(&b_full[sb]), (T / SB) & 1, sm.abort_flag, 39)) {
                  alive = false;
                  break;
                }
                fence_after();
                const uint64_t arow = ap + (uint64_t)(ky * row16);
                const uint64_t brow = bdesc0 + (uint64_t)(sb * stage16);
                if (s0 <= kZsSlots - 3)
                  zs_row<OP, 3>(tmem, dslot, arow, brow);
                else if (s0 == kZsSlots - 2)
                  zs_row<OP, 2>(tmem, dslot, arow, brow);
                else
                  zs_row<OP, 1>(tmem, dslot, arow, brow);
                mma_commit(smem_u32(&b_empty[sb]));
                ++T;
              }
            }
          }
          if (!alive) break;
          mma_commit(smem_u32(&a_empty[sa]));
          ++PA;
          mma_commit(smem_u32(&accf[zs_slot(Pn - 2)]));  // plane u - 1 is complete
        }
        if (!alive) break;
        const int Pl = P + (sg.ub - sg.ua) + 2;  // plane ub + 1
        mma_commit(smem_u32(&accf[zs_slot(Pl - 1)]));
        mma_commit(smem_u32(&accf[zs_slot(Pl)]));
        P = Pl + 1;
      }
      if (*sm.abort_flag) {
        mma_commit(drain_bar);
        mbar_wait(drain_bar, 0, sm.abort_flag, 16, false);
      }
    }
    __syncwarp();
  } else if (warp >= 10) {
    // ----------------------- operand transform (2 warps) ----------------------
    const int t = threadIdx.x - 10 * 32;
    int PA = 0, cur_b = -1;
    bool alive = true, over = false;
    ZsRun run = zs_run(g, (int)blockIdx.x, (int)gridDim.x);
    ZsSegment sg;
    while (alive && zs_next(g, run, sg, (int)blockIdx.x, (int)gridDim.x)) {
      const int b = sg.col / bricks, rem = sg.col - b * bricks;
      const int hb = rem / g.nw, wb = rem - hb * g.nw;
      const int w0 = wb * kHaloW - 1, h0 = hb * kHaloH - 1;
      if (b != cur_b) {
        zs_load_affine(a, g, b, aff, lane);
        cur_b = b;
      }
      for (int u = sg.ua; u <= sg.ub; ++u, ++PA) {
        const int sa = PA % SA;
        // lane 0 waits (bounded) and the warp follows its verdict, so the warp never splits
        int ok = 1;
        if (lane == 0) ok = mbar_wait(smem_u32(&a_full[sa]), (PA / SA) & 1, sm.abort_flag, 41) ? 1 : 0;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          alive = false;
          break;
        }
        mbar_try_wait(smem_u32(&a_full[sa]), (PA / SA) & 1);  // completed phase: acquire for every lane
        for (int c = 0; c < g.nchunk; ++c) {
          const nnb_segment& seg = a.seg[c * BK >= g.c0len ? 1 : 0];
          if (seg.prepared) continue;  // already [hi | lo] rows
          const bool lazy_leaky = seg.scale != nullptr && seg.leaky;
          over |= zs_transform_plane<OP>(a_ring + sa * a_entry + c * g.plane_bytes, g, aff + 64 * c, lazy_leaky,
                                         w0, h0, a.slope, t);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> MMA reads
        __syncwarp();
        if ((t & 31) == 0) mbar_arrive(smem_u32(&a_ready[sa]));
      }
    }
    if (over) atomicAdd(g.range_events, 1ull);
  } else {
    // ------------------------------ epilogue ---------------------------------
    // group 0 (warps 2-5) takes the even planes of the sequence, group 1 (warps 6-9) the odd ones
    const int q = warp & 3;
    const int grp = warp >= 6 ? 1 : 0;
    const int bar = 1 + grp;
    volatile int* votes = grp ? sm.votes2 : sm.votes;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    const float* col_inv = reinterpret_cast<const float*>(wimg + (int64_t)g.ksteps * C::kBBytes);
    const RowPos rp = row_pos(g, q, lane);
    int P = 0;
    ZsRun run = zs_run(g, (int)blockIdx.x, (int)gridDim.x);
    ZsSegment sg;
    bool stop = false;
    while (!stop && zs_next(g, run, sg, (int)blockIdx.x, (int)gridDim.x)) {
      const int b = sg.col / bricks, rem = sg.col - b * bricks;
      const int hb = rem / g.nw, wb = rem - hb * g.nw;
      for (int z = sg.ua - 1; z <= sg.ub + 1; ++z, ++P) {
        if ((P & 1) != grp) continue;
        const int slot = zs_slot(P);
        const bool ok = mbar_wait(smem_u32(&accf[slot]), (P / kZsSlots) & 1, sm.abort_flag, 40);
        if (lane == 0) votes[q] = (!ok || *sm.abort_flag) ? 1 : 0;
        asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
        stop = votes[0] | votes[1] | votes[2] | votes[3];
        asm volatile("bar.sync %0, 128;" ::"r"(bar) : "memory");
        if (stop) break;
        fence_after();
        const uint32_t acc = tmem + lane_base + 32u * (uint32_t)slot;
        if (z >= sg.z0 && z < sg.z1) {
          TileOrigin o;
          o.b = b;
          o.nt = 0;
          o.t = (z * g.nh + hb) * g.nw + wb;
          o.d0 = z;
          o.h0 = hb * kHaloH;
          o.w0 = wb * kHaloW;
          epilogue_tile<BC, OP>(a, g, o, rp, acc, 0u, lane, col_inv, zs_stg + 4 * grp * (kStagingBytes / 16),
                                (warp - 2) & 3, bar);
        }
        tmem_zero32(acc);
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&acce[slot]));
      }
    }
  }
  __syncthreads();
  if (warp == 1) tmem_free_all(tmem);
}

// ---------------------------------------------------------------------------
// Weight image: [n_tile][kstep = chunk * taps + tap][N rows][row bytes] (so
// the taps of one 32-channel chunk are contiguous), natural K order within the
// 32-channel step.  GEMM column n is output channel n, or for a transposed
// convolution (row_taps > 1) the pair (tap = n / up_cout, channel = n % up_cout)
// reading weight (channel, tap, ci).
//   TF32 formats: 128-byte rows, 16-byte chunks XOR-swizzled by row % 8 (the
//   SW128 K-major layout); rows [0, BC) W_hi of the tile's BC columns and rows
//   [BC, 2 BC) W_lo (kOperandTf32x2), or BC rows of TF32.
//   kOperandF16x2: 64-byte rows of halves, 16-byte chunks XOR-swizzled by
//   (row / 2) % 4 (the SW64 K-major layout); rows [0, BC) W0 = fp16(s w), rows
//   [BC, 2 BC) W1 = fp16(s w - W0); after the tiles, 1/s of every column
//   (n_tiles * BC floats).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float weight_at(const float* __restrict__ w, int col, int tap, int ci, int kvol,
                                           int cin_total, int row_taps, int up_cout) {
  if (row_taps > 1) {
    const int co = col % up_cout, utap = col / up_cout;
    return w[((int64_t)co * row_taps + utap) * cin_total + ci];
  }
  return w[((int64_t)col * kvol + tap) * cin_total + ci];
}

__global__ void pack_kernel(const float* __restrict__ w, int cols_total, int kvol, int cin_total, int bc,
                            int halves, int nchunk, int row_taps, int up_cout, int64_t total_words,
                            uint32_t* __restrict__ out) {
  const int nrows = halves * bc;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total_words;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int word = (int)(o % 32);  // 4-byte word within the 128-byte row (physical position)
    int64_t r = o / 32;
    const int n = (int)(r % nrows);
    r /= nrows;
    const int ks = (int)(r % ((int64_t)kvol * nchunk));
    const int nt = (int)(r / ((int64_t)kvol * nchunk));
    const int k = ((word >> 2) ^ (n & 7)) * 4 + (word & 3);
    const int half = n / bc;
    const int col = nt * bc + (n - half * bc);
    const int chunk = ks / kvol, tap = ks - chunk * kvol;  // chunk-major K-step order
    const int ci = chunk * BK + k;
    float val = 0.f;
    if (col < cols_total && ci < cin_total) val = weight_at(w, col, tap, ci, kvol, cin_total, row_taps, up_cout);
    uint32_t res;
    if (halves == 2) {
      const uint32_t hi = __float_as_uint(val) & 0xFFFFE000u;
      res = half == 0 ? hi : __float_as_uint(val - __uint_as_float(hi));
    } else {
      res = to_tf32(val);
    }
    out[o] = res;
  }
}

// 1/s per GEMM column for the fp16-pair image: s = 2^(14 - e) with max |w| =
// f 2^e, f in [0.5, 1), so max |s w| < 2^14 (W0 stays far from fp16 overflow
// and small weights stay normal); all-zero or padding columns get s = 1.
__global__ void column_scale_kernel(const float* __restrict__ w, int cols_total, int kvol, int cin_total,
                                    int row_taps, int up_cout, float* __restrict__ inv_scale) {
  const int col = blockIdx.x;
  float m = 0.f;
  if (col < cols_total) {
    const int64_t K = (int64_t)kvol * cin_total;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
      const int tap = (int)(k / cin_total), ci = (int)(k - (int64_t)tap * cin_total);
      m = fmaxf(m, fabsf(weight_at(w, col, tap, ci, kvol, cin_total, row_taps, up_cout)));
    }
  }
  __shared__ float part[32];
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, part[i]);
    float inv = 1.f;
    if (m > 0.f && isfinite(m)) {
      int e = 0;
      frexpf(m, &e);
      inv = ldexpf(1.f, max(-100, min(100, e - 14)));
    }
    inv_scale[col] = inv;
  }
}

__global__ void pack_f16x2_kernel(const float* __restrict__ w, int cols_total, int kvol, int cin_total, int bc,
                                  int nchunk, int row_taps, int up_cout, int64_t total_words,
                                  const float* __restrict__ inv_scale, uint32_t* __restrict__ out) {
  const int nrows = 2 * bc;
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total_words;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int word = (int)(o % 16);  // 4-byte word (two halves) within the 64-byte row (physical position)
    int64_t r = o / 16;
    const int n = (int)(r % nrows);
    r /= nrows;
    const int ks = (int)(r % ((int64_t)kvol * nchunk));
    const int nt = (int)(r / ((int64_t)kvol * nchunk));
    const int k = (((word >> 2) ^ ((n >> 1) & 3)) * 4 + (word & 3)) * 2;  // first of the word's two channels
    const int half = n / bc;
    const int col = nt * bc + (n - half * bc);
    const int chunk = ks / kvol, tap = ks - chunk * kvol;
    const float s = 1.f / __ldg(inv_scale + nt * bc + (n - half * bc));  // exact: a power of two
    uint32_t res = 0;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int ci = chunk * BK + k + e;
      float val = 0.f;
      if (col < cols_total && ci < cin_total) val = weight_at(w, col, tap, ci, kvol, cin_total, row_taps, up_cout) * s;
      const __half h0 = __float2half_rn(val);
      const __half h = half == 0 ? h0 : __float2half_rn(val - __half2float(h0));
      res |= (uint32_t)__half_as_ushort(h) << (16 * e);
    }
    out[o] = res;
  }
}

// bf16 image: 64-byte rows of bf16(w) (round to nearest even), SW64 like the fp16-pair image, BC rows per
// K-step and no column scales (bf16 keeps float32's exponent range).
__global__ void pack_bf16_kernel(const float* __restrict__ w, int cols_total, int kvol, int cin_total, int bc,
                                 int nchunk, int row_taps, int up_cout, int64_t total_words,
                                 uint32_t* __restrict__ out) {
  for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total_words;
       o += (int64_t)gridDim.x * blockDim.x) {
    const int word = (int)(o % 16);  // 4-byte word (two bf16) within the 64-byte row (physical position)
    int64_t r = o / 16;
    const int n = (int)(r % bc);
    r /= bc;
    const int ks = (int)(r % ((int64_t)kvol * nchunk));
    const int nt = (int)(r / ((int64_t)kvol * nchunk));
    const int k = (((word >> 2) ^ ((n >> 1) & 3)) * 4 + (word & 3)) * 2;  // first of the word's two channels
    const int col = nt * bc + n;
    const int chunk = ks / kvol, tap = ks - chunk * kvol;
    uint32_t res = 0;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int ci = chunk * BK + k + e;
      float val = 0.f;
      if (col < cols_total && ci < cin_total) val = weight_at(w, col, tap, ci, kvol, cin_total, row_taps, up_cout);
      res |= (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(val)) << (16 * e);
    }
    out[o] = res;
  }
}

// Bytes of one B tile (one K-step of BC columns) in the operand format.
inline int b_tile_bytes(int op, int bc) {
  return op == kOperandF16x2 ? 2 * bc * 64 : op == kOperandBf16 ? bc * 64 : op == kOperandTf32x2 ? 2 * bc * 128 : bc * 128;
}

inline int pick_bc(int cols) {
  if (cols <= 32) return 32;
  if (cols <= 64) return 64;
  return 128;
}

// Brick (tw, th, td) with tw*th*td <= 128 covering the row space with the
// fewest tiles (ties: the widest rows); a strided box spans tw * stride <= 256.
inline void choose_brick(const int od, const int oh, const int ow, const int sd, const int sh, const int sw,
                         int& tw, int& th, int& td) {
  int64_t best = INT64_MAX;
  tw = th = td = 1;
  const int mw = std::min({ow, BM, 256 / sw});
  for (int w = mw; w >= 1; --w) {
    const int mh = std::min({oh, BM / w, 256 / sh});
    for (int h = mh; h >= 1; --h) {
      const int d = std::min({od, BM / (w * h), 256 / sd});
      const int64_t tiles = (int64_t)((ow + w - 1) / w) * ((oh + h - 1) / h) * ((od + d - 1) / d);
      if (tiles < best) {
        best = tiles;
        tw = w;
        th = h;
        td = d;
      }
    }
  }
}

// Halo mode when the layer is a unit-stride multi-tap conv over at least one
// 8-wide brick row, <= 64 output channels per tile, and two A planes plus four
// B tiles fit the shared-memory budget.  halves: A boxes per chunk; bbytes:
// bytes of one B tile.
inline bool plan_halo(const nnb_conv3d_args& a, Geometry& g, int halves, int bbytes) {
  if (g.SD != 1 || g.SH != 1 || g.SW != 1) return false;
  if (g.KD * g.KH * g.KW < 2 || g.OW < kHaloW || g.OH < kHaloH / 2) return false;
  if (pick_bc(a.cout) > 64) return false;
  g.pw = kHaloW + g.KW - 1;
  const int ph = kHaloH + g.KH - 1;
  if (g.pw > 256 || ph > 256) return false;
  g.plane_rows = g.pw * ph;
  g.plane_bytes = (g.plane_rows * 128 + 1023) & ~1023;
  const int a_stage = halves * g.plane_bytes;
  const int budget = kMaxSmem - 1024 - kMiscBytes - 8 * kStagingBytes;
  // Ring plan, first that fits: B stages of a whole kx row (3-wide kernels) with 3 A planes and
  // >= 3 B stages, then with 2 A planes and >= 2 B stages, else one tap per B stage.
  if (g.KW == 3 && 3 * a_stage + 3 * 3 * bbytes <= budget) {
    g.sa = 3;
    g.tb = 3;
  } else if (g.KW == 3 && 2 * a_stage + 2 * 3 * bbytes <= budget) {
    g.sa = 2;
    g.tb = 3;
  } else {
    g.sa = (3 * a_stage + 4 * bbytes <= budget) ? 3 : 2;
    g.tb = 1;
  }
  g.sb = std::min(16, (budget - g.sa * a_stage) / (g.tb * bbytes));
  if (g.sb < (g.tb > 1 ? 2 : 4) || 2 * g.sa + 2 * g.sb + 5 > kMaxBars) return false;
  g.box[0] = g.pw;
  g.box[1] = ph;
  g.box[2] = 1;
  g.tw = kHaloW;
  g.th = kHaloH;
  g.td = 1;
  return true;
}

// Z-streaming mode (fp16 pairs, bf16 or TF32) when the layer is a 3x3x3,
// stride-1, padding-1 conv with <= 32 output channels over at least one
// 8-wide brick row, and the A ring plus the weights (resident for one
// 32-channel chunk, else >= 2 streamed (chunk, ky) stages) fit the
// shared-memory budget.
inline bool plan_zstream(const nnb_conv3d_args& a, Geometry& g, int op) {
  if (a.operand_format != 2 || pick_bc(a.cout) != 32) return false;
  if (op != kOperandF16x2 && op != kOperandBf16 && op != kOperandTf32) return false;
  for (int i = 0; i < 3; ++i)
    if (a.kernel[i] != 3 || a.stride[i] != 1 || a.pad[i] != 1) return false;
  if (g.OW < kHaloW || g.OH < kHaloH / 2 || g.nchunk < 1) return false;
  g.pw = kHaloW + 2;
  const int ph = kHaloH + 2;
  g.plane_rows = g.pw * ph;
  g.plane_bytes = (g.plane_rows * 128 + 1023) & ~1023;
  const int entry = g.nchunk * g.plane_bytes;
  const int budget = kMaxSmem - 1024 - kMiscBytes - 2 * g.nchunk * 64 * 4 - 8 * kStagingBytes;  // tables, staging
  const int tap_bytes = zs_tap_bytes(op);
  if (2 * entry + g.nchunk * 9 * tap_bytes <= budget) {
    // every chunk's weights resident (one chunk of any format; two chunks of the bf16 format)
    g.sb = 0;
    g.sa = std::min(4, (budget - g.nchunk * 9 * tap_bytes) / entry);
  } else {
    g.sa = 2;
    g.sb = std::min(4, (budget - 2 * entry) / (3 * tap_bytes));
    if (g.sb < 2) return false;
  }
  if (3 * g.sa + 2 * std::max(g.sb, 1) + 2 * kZsSlots + 1 > kMaxBars) return false;
  g.box[0] = g.pw;
  g.box[1] = ph;
  g.box[2] = 1;
  g.tw = kHaloW;
  g.th = kHaloH;
  g.td = 1;
  g.tb = 3;
  g.halo = 1;  // plane boxes with unit element strides
  g.zs = 1;
  return true;
}

// Row-space geometry shared by the launch, the weight image size and the
// partials query.
inline Geometry make_geometry(const nnb_conv3d_args& a) {
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
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) cin_total += a.seg[s].channels;
  g.c0len = a.seg[0].channels;
  g.nchunk = cin_total / BK;
  g.ksteps = g.KD * g.KH * g.KW * g.nchunk;
  const int bc = pick_bc(a.cout);
  g.n_tiles = (a.cout + bc - 1) / bc;
  g.up_cout = 0;
  const int op = operand_kind(a.precision);
  g.zs = 0;
  if (!plan_zstream(a, g, op)) g.halo = plan_halo(a, g, op == kOperandTf32x2 ? 2 : 1, b_tile_bytes(op, bc)) ? 1 : 0;
  if (!g.halo) {
    choose_brick(g.OD, g.OH, g.OW, g.SD, g.SH, g.SW, g.tw, g.th, g.td);
    g.box[0] = g.tw * g.SW;
    g.box[1] = g.th * g.SH;
    g.box[2] = g.td * g.SD;
  }
  g.rows = g.tw * g.th * g.td;
  g.nw = (g.OW + g.tw - 1) / g.tw;
  g.nh = (g.OH + g.th - 1) / g.th;
  g.tps = g.nw * g.nh * ((g.OD + g.td - 1) / g.td);
  return g;
}

using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

inline EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 5-D map (elements per voxel, W, H, D, batch) of one prepared operand; the box
// is one 128-byte row (32 floats, or 64 halves = [hi | lo] of 32 channels) x
// the mode's box extent, sampled every stride voxels.
inline int encode_operand(const nnb_segment& seg, int op, int batch, const Geometry& g, CUtensorMap* map) {
  const EncodeTiledFn fn = encode_tiled();
  NNB_REQUIRE(fn != nullptr, "conv3d: cuTensorMapEncodeTiled is not available from the driver");
  // z-streaming mode loads the raw float32 activation, or a segment already prepared as fp16 pairs
  const bool raw = g.zs && !seg.prepared;
  const bool f16 = half_rows(op) && !raw;  // 16-bit rows (fp16 pair or bf16), copied bit for bit
  const cuuint64_t inner = (cuuint64_t)(op == kOperandTf32 || raw ? 1 : 2) * seg.channels;
  const cuuint64_t esize = f16 ? 2 : 4;
  const cuuint64_t dims[5] = {inner, (cuuint64_t)g.IW, (cuuint64_t)g.IH, (cuuint64_t)g.ID, (cuuint64_t)batch};
  const cuuint64_t row = inner * esize;
  const cuuint64_t strides[4] = {row, row * g.IW, row * g.IW * g.IH, row * g.IW * g.IH * g.ID};
  const cuuint32_t box[5] = {(cuuint32_t)(128 / esize), (cuuint32_t)g.box[0], (cuuint32_t)g.box[1],
                             (cuuint32_t)g.box[2], 1u};
  const cuuint32_t estr[5] = {1u, (cuuint32_t)(g.halo ? 1 : g.SW), (cuuint32_t)(g.halo ? 1 : g.SH),
                              (cuuint32_t)(g.halo ? 1 : g.SD), 1u};
  const CUresult r = fn(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5,
                        const_cast<float*>(seg.data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  NNB_REQUIRE(r == CUDA_SUCCESS, "conv3d: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return NNB_OK;
}

template <int BC, int OP>
int launch_bc(const nnb_conv3d_args& a, const Geometry& g, const OperandMaps& maps, cudaStream_t stream) {
  using C = Cfg<BC, OP>;
  int dev = 0;
  NNB_CUDA_CHECK(cudaGetDevice(&dev));
  static int configured[64] = {0};  // dynamic shared memory opt-in done (bit 0 box, 1/2 halo TB 1/3, 3+ zs per OP)
  const int bit = g.zs ? (8 << OP) : g.halo ? (g.tb == 3 ? 4 : 2) : 1;
  if (dev >= 64 || !(configured[dev] & bit)) {
    if (g.zs) {
      if constexpr (BC == 32 && (OP == kOperandF16x2 || OP == kOperandBf16 || OP == kOperandTf32))
        NNB_CUDA_CHECK(cudaFuncSetAttribute(conv3d_zstream_kernel<OP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kMaxSmem));
    } else if (g.halo && g.tb == 3)
      NNB_CUDA_CHECK(cudaFuncSetAttribute(conv3d_halo_kernel<BC, OP, 3>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    else if (g.halo)
      NNB_CUDA_CHECK(cudaFuncSetAttribute(conv3d_halo_kernel<BC, OP, 1>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    else
      NNB_CUDA_CHECK(cudaFuncSetAttribute(conv3d_tc_kernel<BC, OP>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem));
    if (dev < 64) configured[dev] |= bit;
  }
  int sms = 148;
  NNB_CUDA_CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int grid = std::min(g.total_tiles, sms);
  if (g.zs) {
    if constexpr (BC == 32 && (OP == kOperandF16x2 || OP == kOperandBf16 || OP == kOperandTf32)) {
      const int b_bytes = g.sb == 0 ? g.nchunk * 9 * zs_tap_bytes(OP) : g.sb * 3 * zs_tap_bytes(OP);
      const int smem = 1024 + g.sa * g.nchunk * g.plane_bytes + b_bytes + kMiscBytes + 2 * g.nchunk * 64 * 4 +
                       8 * kStagingBytes;
      NNB_REQUIRE(smem <= kMaxSmem, "conv3d: z-streaming plan exceeds shared memory (%d bytes)", smem);
      conv3d_zstream_kernel<OP><<<grid, kZsThreads, smem, stream>>>(a, g, maps);
    } else {
      NNB_REQUIRE(false, "conv3d: internal: z-streaming plan for an unsupported tile");
    }
  } else if (g.halo) {
    const int smem = 1024 + g.sa * C::kHalves * g.plane_bytes + g.sb * g.tb * C::kBBytes + kMiscBytes +
                     8 * kStagingBytes;
    NNB_REQUIRE(smem <= kMaxSmem, "conv3d: halo plan exceeds shared memory (%d bytes)", smem);
    if (g.tb == 3)
      conv3d_halo_kernel<BC, OP, 3><<<grid, C::kThreadsC, smem, stream>>>(a, g, maps);
    else
      conv3d_halo_kernel<BC, OP, 1><<<grid, C::kThreadsC, smem, stream>>>(a, g, maps);
  } else {
    const int smem = 1024 + C::S * C::kStageBytes + kMiscBytes + 4 * kMaxKsteps + 8 * kStagingBytes;
    conv3d_tc_kernel<BC, OP><<<grid, C::kThreadsC, smem, stream>>>(a, g, maps);
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int dispatch(const nnb_conv3d_args& a, Geometry& g, cudaStream_t stream) {
  const int64_t tiles = (int64_t)a.batch * g.tps * g.n_tiles;
  NNB_REQUIRE(tiles < (1LL << 31), "conv3d: too many tiles");
  g.total_tiles = (int)tiles;
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(a.packed) & 1023) == 0, "conv3d: packed weights must be 1024-aligned");
  const int op = operand_kind(a.precision);
  OperandMaps maps;
  for (int s = 0; s < a.num_segments; ++s) {
    const int rc = encode_operand(a.seg[s], op, a.batch, g, &maps.seg[s]);
    if (rc) return rc;
  }
  if (a.num_segments == 1) maps.seg[1] = maps.seg[0];
  const int bc = pick_bc(a.cout);
  NNB_REQUIRE(bc <= 64 || !g.halo, "conv3d: internal: halo plan for a 128-column tile");
  switch (op * 4 + (bc == 32 ? 0 : bc == 64 ? 1 : 2)) {
    case kOperandF16x2 * 4 + 0: return launch_bc<32, kOperandF16x2>(a, g, maps, stream);
    case kOperandF16x2 * 4 + 1: return launch_bc<64, kOperandF16x2>(a, g, maps, stream);
    case kOperandF16x2 * 4 + 2: return launch_bc<128, kOperandF16x2>(a, g, maps, stream);
    case kOperandTf32x2 * 4 + 0: return launch_bc<32, kOperandTf32x2>(a, g, maps, stream);
    case kOperandTf32x2 * 4 + 1: return launch_bc<64, kOperandTf32x2>(a, g, maps, stream);
    case kOperandTf32x2 * 4 + 2: return launch_bc<128, kOperandTf32x2>(a, g, maps, stream);
    case kOperandBf16 * 4 + 0: return launch_bc<32, kOperandBf16>(a, g, maps, stream);
    case kOperandBf16 * 4 + 1: return launch_bc<64, kOperandBf16>(a, g, maps, stream);
    case kOperandBf16 * 4 + 2: return launch_bc<128, kOperandBf16>(a, g, maps, stream);
    case kOperandTf32 * 4 + 0: return launch_bc<32, kOperandTf32>(a, g, maps, stream);
    case kOperandTf32 * 4 + 1: return launch_bc<64, kOperandTf32>(a, g, maps, stream);
    default: return launch_bc<128, kOperandTf32>(a, g, maps, stream);
  }
}

}  // namespace tc

unsigned long long* operand_range_events_ptr();

bool conv3d_tc_supported(const nnb_conv3d_args& a) {
  if (!tensor_precision(a.precision)) return false;
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) {
    if (a.seg[s].channels % tc::BK != 0) return false;
    if ((reinterpret_cast<uintptr_t>(a.seg[s].data) & 15) != 0) return false;
    cin_total += a.seg[s].channels;
  }
  if (a.cout % 16 != 0) return false;
  for (int i = 0; i < 3; ++i) {
    if (a.kernel[i] > 15 || a.stride[i] > 8) return false;  // 4-bit tap offsets; TMA element strides <= 8
  }
  // K-step table capacity (taps x 32-channel chunks)
  return (int64_t)a.kernel[0] * a.kernel[1] * a.kernel[2] * (cin_total / tc::BK) <= tc::kMaxKsteps;
}

int64_t conv3d_tc_packed_bytes(int cols, int kvol, int cin_total, int precision) {
  if (cols < 1 || kvol < 1 || cin_total < 1 || cin_total % tc::BK != 0) return 0;
  if (!tensor_precision(precision)) return 0;
  const int op = operand_kind(precision);
  const int bc = tc::pick_bc(cols);
  const int n_tiles = (cols + bc - 1) / bc;
  const int64_t tiles = (int64_t)n_tiles * kvol * (cin_total / tc::BK) * tc::b_tile_bytes(op, bc);
  return tiles + (op == kOperandF16x2 ? (int64_t)n_tiles * bc * (int64_t)sizeof(float) : 0);
}

int launch_conv3d_pack_rows(const float* w, int cols, int kvol, int cin_total, int precision, int row_taps,
                            int up_cout, void* packed, cudaStream_t stream) {
  NNB_REQUIRE(cin_total % tc::BK == 0, "pack: input channels must be a multiple of %d", tc::BK);
  NNB_REQUIRE(tensor_precision(precision), "pack: precision %d has no weight image", precision);
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(packed) & 1023) == 0, "pack: image must be 1024-byte aligned");
  const int op = operand_kind(precision);
  const int bc = tc::pick_bc(cols);
  const int n_tiles = (cols + bc - 1) / bc;
  const int nchunk = cin_total / tc::BK;
  const int64_t tile_bytes = (int64_t)n_tiles * kvol * nchunk * tc::b_tile_bytes(op, bc);
  const int64_t words = tile_bytes / 4;
  const int blocks = (int)std::min<int64_t>((words + 255) / 256, 148 * 32);
  if (op == kOperandBf16) {
    tc::pack_bf16_kernel<<<blocks, 256, 0, stream>>>(w, cols, kvol, cin_total, bc, nchunk, row_taps, up_cout, words,
                                                     reinterpret_cast<uint32_t*>(packed));
  } else if (op == kOperandF16x2) {
    float* inv_scale = reinterpret_cast<float*>(static_cast<uint8_t*>(packed) + tile_bytes);
    tc::column_scale_kernel<<<n_tiles * bc, 256, 0, stream>>>(w, cols, kvol, cin_total, row_taps, up_cout,
                                                               inv_scale);
    NNB_LAUNCH_CHECK();
    tc::pack_f16x2_kernel<<<blocks, 256, 0, stream>>>(w, cols, kvol, cin_total, bc, nchunk, row_taps, up_cout, words,
                                                      inv_scale, reinterpret_cast<uint32_t*>(packed));
  } else {
    const int halves = op == kOperandTf32x2 ? 2 : 1;
    tc::pack_kernel<<<blocks, 256, 0, stream>>>(w, cols, kvol, cin_total, bc, halves, nchunk, row_taps, up_cout,
                                                words, reinterpret_cast<uint32_t*>(packed));
  }
  NNB_LAUNCH_CHECK();
  return NNB_OK;
}

int launch_conv3d_pack(const float* w, int cout, int kvol, int cin_total, int precision, void* packed,
                       cudaStream_t stream) {
  return launch_conv3d_pack_rows(w, cout, kvol, cin_total, precision, 1, cout, packed, stream);
}

// Whether the tensor-core path reads raw lazy segments for these shapes (z-streaming mode).
bool conv3d_tc_raw_operands(const nnb_conv3d_args& a) {
  if (a.precision != NNB_PREC_FP32 && a.precision != NNB_PREC_BF16 && a.precision != NNB_PREC_TF32) return false;
  if (!(a.slope >= 0.f && a.slope <= 1.f)) return false;
  int cin_total = 0;
  for (int s = 0; s < a.num_segments; ++s) {
    if (a.seg[s].channels % tc::BK != 0) return false;
    cin_total += a.seg[s].channels;
  }
  if (a.cout % 16 != 0 || 27 * (cin_total / tc::BK) > tc::kMaxKsteps) return false;
  nnb_conv3d_args r = a;
  r.operand_format = 2;
  return tc::make_geometry(r).zs == 1;
}

// Tiles per sample of the partials a tensor-core convolution writes.
int conv3d_tc_partial_tiles(const nnb_conv3d_args& a) { return tc::make_geometry(a).tps; }

// Kernel a tensor-core convolution launches: 1 box, 2 halo, 3 z-streaming.
int conv3d_tc_mode(const nnb_conv3d_args& a) {
  const tc::Geometry g = tc::make_geometry(a);
  return g.zs ? 3 : g.halo ? 2 : 1;
}

int launch_conv3d_tc(const nnb_conv3d_args& a, cudaStream_t stream) {
  tc::Geometry g = tc::make_geometry(a);
  if (g.zs) {
    g.range_events = operand_range_events_ptr();
    NNB_REQUIRE(g.range_events != nullptr, "conv3d: range-event counter unavailable");
  }
  NNB_REQUIRE(a.operand_format != 2 || g.zs, "conv3d: raw tensor-core operands outside the z-streaming envelope");
  return tc::dispatch(a, g, stream);
}

// Stride == kernel transposed convolution as a 1x1x1 GEMM (rows = input
// voxels, N = taps x cout) with the scatter epilogue.
int launch_conv_transpose_tc(const nnb_segment& in, int batch, const int32_t in_dims[3], const int32_t k[3],
                             float slope, const float* bias, int cout, const void* packed, int precision, float* out,
                             int out_operand, cudaStream_t stream) {
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
  NNB_REQUIRE((reinterpret_cast<uintptr_t>(bias) & 15) == 0, "conv_transpose3d: bias must be 16-byte aligned");
  NNB_REQUIRE(conv3d_tc_supported(a) && cout % 32 == 0, "conv_transpose3d: outside the tensor-core envelope");
  tc::Geometry g = tc::make_geometry(a);
  g.up_cout = cout;
  g.UKD = k[0];
  g.UKH = k[1];
  g.UKW = k[2];
  g.up_operand = out_operand;
  if (out_operand) {
    NNB_REQUIRE(precision == NNB_PREC_FP32 || precision == NNB_PREC_BF16 || precision == NNB_PREC_TF32,
                "conv_transpose3d: operand output needs NNB_PREC_FP32, NNB_PREC_BF16 or NNB_PREC_TF32");
    g.range_events = operand_range_events_ptr();
    NNB_REQUIRE(g.range_events != nullptr, "conv_transpose3d: range-event counter unavailable");
  }
  return tc::dispatch(a, g, stream);
}

}  // namespace nnb

extern "C" int32_t nnb_device_status(int32_t* where, int32_t reset) {
  int status = 0, loc = 0;
  if (cudaDeviceSynchronize() != cudaSuccess) return NNB_E_CUDA;
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
