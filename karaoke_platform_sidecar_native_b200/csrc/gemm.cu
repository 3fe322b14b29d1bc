// Persistent tcgen05 GEMM for sm_100a:  C[M][N] = A[M][K] * B[N][K]^T, and
// (ffn_kernel, further down) the fused feed-forward sub-block of a width-256
// row, FF1 -> GELU -> FF2 + residual with the hidden kept on chip.
//
// One CTA per SM walks a static tile schedule.  Warp 0 issues TMA loads of
// 128x64 A and (n_size)x64 B tiles into a 3-stage 128-byte-swizzled ring, warp
// 1 (one thread) issues tcgen05.mma (M=128, N=n_size<=256, K=16) into one of
// two TMEM accumulators, and warps 2-9 (two per TMEM lane quarter, each owning
// 128 columns) drain the other accumulator with tcgen05.ld.
//
// Epilogue I/O is staged: each epilogue warp writes its 32-row block into a
// swizzled shared-memory buffer and a TMA tensor store moves it to global
// memory (and the fp32 residual comes in by TMA load the same way), so global
// traffic is whole lines instead of one row per thread.
//
// RMSNorm is folded: the gamma of the norm that precedes a GEMM is multiplied
// into that GEMM's weights at load time, the producer of x writes a 16-bit copy
// of x and the per-row factor inv = sqrt(256) / sqrt(sum x^2 + 1e-12), and the
// consumer scales its accumulator row by inv:  (x * inv * gamma) W^T =
// inv * (x (gamma o W)^T).  The head gates (Linear 256 -> 8 of the normed row)
// are the 16-column tail tile of the QKV GEMM.
//
// The reference computes these products with cuBLAS SGEMM plus separate SIMT
// kernels (native/native_gpu_cuda.cu:540-552, :258-297, :403-426, :453-485);
// the CPU semantics are transformer_forward (native/vocalarc_separation.c:836-873).
#include <cstdio>

#include "ptx.cuh"
#include "vab_internal.h"

namespace vab {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 3;
constexpr int kABytes = kBM * kBK * 2;   // 16 KB
constexpr int kBBytes = kBN * kBK * 2;   // 32 KB
constexpr int kThreads = 320;            // TMA warp, MMA warp, 8 epilogue warps
constexpr int kEpiWarps = 8;
constexpr int kTmemCols = 512;           // two 128x256 fp32 accumulators
constexpr int kStageBuf = 4096;          // one epilogue staging buffer: 32 rows x 128 B
constexpr int kRedBytes = 2 * 2 * 128 * 4;
constexpr int kBarBytes = 512;
constexpr int kSmemBytes =
    1024 + kStages * (kABytes + kBBytes) + kEpiWarps * 2 * kStageBuf + kRedBytes + kBarBytes;

__constant__ int c_band_first[kBands];
__constant__ int c_band_dim[kBands];

struct TileInfo {
  int a_row, b_row, n0, m_valid, n_size, band;
};

__device__ __forceinline__ TileInfo decode_tile(const GemmArgs& args, int tile) {
  TileInfo t;
  if (args.tiles == nullptr) {
    const int per_m = args.n_tiles + (args.gate_tile ? 1 : 0);
    const int m_blk = tile / per_m;
    const int n_blk = tile - m_blk * per_m;
    t.a_row = m_blk * kBM;
    t.m_valid = min(kBM, args.m_rows - t.a_row);
    t.b_row = n_blk * kBN;
    t.n0 = n_blk * kBN;
    t.n_size = n_blk < args.n_tiles ? kBN : 16;   // the gate tile: 8 gate rows + 8 zero rows
    t.band = 0;
  } else {
    const int chunk = tile / args.tiles_per_chunk;
    const int4 e = args.tiles[tile - chunk * args.tiles_per_chunk];
    t.a_row = e.x + chunk * args.chunk_rows;
    t.b_row = e.y;
    t.n0 = e.z;
    t.m_valid = e.w & 0xFF;
    t.n_size = (e.w >> 8) & 0x1FF;
    t.band = e.w >> 17;
  }
  return t;
}

// Exact-erf GELU, x * h(x) with h = (1 + erf(x / sqrt 2)) / 2, for a pair of
// values, written as h = (1 + tanh(g(x))) / 2 with g(x) = atanh(erf(x / sqrt 2)),
// a smooth odd function.  g is x (c0 + c1 x^2 + c2 x^4) on |x| <= 4.5
// (coefficients fitted here, minimax in h; |h error| <= 1.9e-5 with an exact
// tanh); beyond it x^2 is clamped to 4.5^2, so g = 1.41 x keeps growing and h
// goes to 0 or 1 (h is within 3.4e-6 of them there).  GELU = x/2 + (x/2) tanh(g)
// as one FMA.  tanh runs on MUFU (tanh.approx.f32; measured on the B200:
// relative error below 2^-16.6), so a value costs one MUFU operation and about
// six FMA-pipe operations instead of the sixteen of a polynomial for erf
// itself, which made the FFN input GEMM's epilogue FMA-bound.  Measured GELU
// error: max 5.5e-5, rms 1.6e-5 absolute -- below the 16-bit rounding of the
// stored hidden.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 gelu_pair(float2 x) {
  const float2 x2 = __fmul2_rn(x, x);
  const float2 s = make_float2(fminf(x2.x, 20.25f), fminf(x2.y, 20.25f));
  float2 p = __ffma2_rn(s, make_float2(-0.00031580726499669254f, -0.00031580726499669254f),
                        make_float2(0.03679825738072395f, 0.03679825738072395f));
  p = __ffma2_rn(p, s, make_float2(0.797717809677124f, 0.797717809677124f));
  const float2 g = __fmul2_rn(p, x);
  const float2 hx = __fmul2_rn(x, make_float2(0.5f, 0.5f));
  return __ffma2_rn(hx, make_float2(tanh_approx(g.x), tanh_approx(g.y)), hx);
}

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + __expf(-x)); }

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Byte offset of 16-byte chunk q of row r in a 128-byte-row, 128B-swizzled buffer.
__device__ __forceinline__ int sw128(int r, int q) { return r * 128 + ((q ^ (r & 7)) << 4); }
// Same for 64-byte rows and the 64B swizzle.
__device__ __forceinline__ int sw64(int r, int q) { return r * 64 + ((q ^ ((r >> 1) & 3)) << 4); }

template <typename T>
__device__ __forceinline__ void store_row16(T* dst, const float* v, int count) {
  // Direct per-row store (grouped mask and test epilogues). count is 16 or 32.
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q * 8 >= count) break;
    uint4 w;
    w.x = ElemTraits<T>::pack2(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = ElemTraits<T>::pack2(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = ElemTraits<T>::pack2(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = ElemTraits<T>::pack2(v[q * 8 + 6], v[q * 8 + 7]);
    d[q] = w;
  }
}

// Per-warp epilogue state: two staging buffers, their TMA-load barriers and phases.
struct EpiWarp {
  uint8_t* buf[2];
  uint64_t* bar[2];
  uint32_t phase[2];
  int cur;
  int lane;
};

// ---------------------------------------------------------------- 16-bit outputs
// QKV (+RoPE, row scale), FF1 (+bias, GELU, row scale), plain store.  This warp
// owns columns [128*half, 128*half + 128) of the tile in two 64-column steps.
// `inv` and `rope` (this row's RMSNorm factor and RoPE cos/sin) are loaded by
// the caller before it waits for the accumulator, so their latency overlaps
// the MMA of the tile.
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_out16(const GemmArgs& args, const CUtensorMap* map_out, const TileInfo& ti,
                                               EpiWarp& ew, uint32_t taddr, int half, int row, int row0, float inv,
                                               const float4 (&rope)[16]) {
  const bool do_rope = EPI == kEpiQkvRope && ti.n0 < args.rope_cols;
#pragma unroll
  for (int s = 0; s < 2; ++s) {
    const int c = half * 128 + s * 64;   // tile column of this step
    uint8_t* buf = ew.buf[ew.cur];
    if (ew.lane == 0) bulk_wait_read1();   // the store that last used this buffer has read it
    __syncwarp();
    const int n = ti.n0 + c;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {   // two 32-column halves of the 64-column step
      uint32_t r[32];
      tmem_ld32(taddr + c + 32 * hh, r);
      tmem_wait_ld();
      reg_fence(r);
      float v[32];
      if (EPI == kEpiGelu || (EPI == kEpiStore && args.bias != nullptr)) {
        // v = acc * inv + bias, two columns per instruction.
        const float2 inv2 = make_float2(inv, inv);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b = __ldg(reinterpret_cast<const float4*>(args.bias + n + 32 * hh) + q);
          const float2 lo = __ffma2_rn(make_float2(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1])), inv2,
                                       make_float2(b.x, b.y));
          const float2 hi = __ffma2_rn(make_float2(__uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])),
                                       inv2, make_float2(b.z, b.w));
          v[4 * q] = lo.x;
          v[4 * q + 1] = lo.y;
          v[4 * q + 2] = hi.x;
          v[4 * q + 3] = hi.y;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * inv;
      }
      if (EPI == kEpiGelu) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          const float2 g = gelu_pair(make_float2(v[j], v[j + 1]));
          v[j] = g.x;
          v[j + 1] = g.y;
        }
      }
      if (do_rope) {
        // A 64-column step is one head: pairs (2i, 2i+1) rotate by rope pair i.
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 cs = rope[8 * hh + i];
          float a = v[4 * i], b = v[4 * i + 1];
          v[4 * i] = a * cs.x - b * cs.y;
          v[4 * i + 1] = a * cs.y + b * cs.x;
          a = v[4 * i + 2];
          b = v[4 * i + 3];
          v[4 * i + 2] = a * cs.z - b * cs.w;
          v[4 * i + 3] = a * cs.w + b * cs.z;
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = ElemTraits<T>::pack2(v[q * 8 + 0], v[q * 8 + 1]);
        w.y = ElemTraits<T>::pack2(v[q * 8 + 2], v[q * 8 + 3]);
        w.z = ElemTraits<T>::pack2(v[q * 8 + 4], v[q * 8 + 5]);
        w.w = ElemTraits<T>::pack2(v[q * 8 + 6], v[q * 8 + 7]);
        *reinterpret_cast<uint4*>(buf + sw128(row & 31, 4 * hh + q)) = w;
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (ew.lane == 0) {
      tma_store_2d(map_out, buf, n, row0);
      bulk_commit();
    }
    ew.cur ^= 1;
  }
}

// ---------------------------------------------------------------- fp32 residual + row statistics
// resid += acc (+ bias); writes resid (fp32), its 16-bit copy and, combined with
// the other column half through shared memory, inv = sqrt(256)/sqrt(sum + 1e-12)
// for the row (transformer_forward's residual_add + the following rms_norm's
// scale, vocalarc_separation.c:864-866, :849, rms_norm_row_scalar :419-424).
// residual_blocks does the four 32-column blocks of this warp's half and
// returns the row's partial sum of squares; the caller combines the halves.
template <typename T>
__device__ __forceinline__ float residual_blocks(const GemmArgs& args, const CUtensorMap* map_res,
                                                 const CUtensorMap* map_x16, int n0, EpiWarp& ew, uint32_t taddr,
                                                 int half, int row, bool valid, int row0) {
  float ss = 0.f;
  // Prefetch the first residual block of this warp's columns.
  if (ew.lane == 0) {
    bulk_wait_read0();
    mbar_arrive_expect_tx(ew.bar[ew.cur], kStageBuf);
    tma_load_2d(ew.buf[ew.cur], map_res, ew.bar[ew.cur], n0 + half * 128, row0);
  }
  __syncwarp();
#pragma unroll 1
  for (int s = 0; s < 4; ++s) {
    const int b = ew.cur;
    const int c = half * 128 + s * 32;
    const int n = n0 + c;
    if (ew.lane == 0 && s + 1 < 4) {
      bulk_wait_read0();   // both stores from the other buffer have read it
      mbar_arrive_expect_tx(ew.bar[b ^ 1], kStageBuf);
      tma_load_2d(ew.buf[b ^ 1], map_res, ew.bar[b ^ 1], n + 32, row0);
    }
    __syncwarp();
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
    reg_fence(r);
    // Bounded wait for the residual block (TMA load issued above).
    {
      const unsigned long long start = global_timer_ns();
      while (!mbar_try_wait(ew.bar[b], ew.phase[b])) {
        if (global_timer_ns() - start > kWaitLimitNs) {
          atomicCAS(args.err, 0, kErrWaitEpilogue);
          break;
        }
      }
    }
    ew.phase[b] ^= 1u;
    uint8_t* buf = ew.buf[b];
    float x[32];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      float4 xv = *reinterpret_cast<const float4*>(buf + sw128(row & 31, q));
      float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (args.bias != nullptr) bv = __ldg(reinterpret_cast<const float4*>(args.bias + n) + q);
      xv.x += __uint_as_float(r[4 * q]) + bv.x;
      xv.y += __uint_as_float(r[4 * q + 1]) + bv.y;
      xv.z += __uint_as_float(r[4 * q + 2]) + bv.z;
      xv.w += __uint_as_float(r[4 * q + 3]) + bv.w;
      x[4 * q] = xv.x;
      x[4 * q + 1] = xv.y;
      x[4 * q + 2] = xv.z;
      x[4 * q + 3] = xv.w;
      *reinterpret_cast<float4*>(buf + sw128(row & 31, q)) = xv;
    }
    if (valid) {
#pragma unroll
      for (int j = 0; j < 32; ++j) ss += x[j] * x[j];
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (ew.lane == 0) {
      tma_store_2d(map_res, buf, n, row0);
      bulk_commit();
      bulk_wait_read0();   // the fp32 block is read out; reuse the buffer for the 16-bit copy
    }
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = ElemTraits<T>::pack2(x[q * 8 + 0], x[q * 8 + 1]);
      w.y = ElemTraits<T>::pack2(x[q * 8 + 2], x[q * 8 + 3]);
      w.z = ElemTraits<T>::pack2(x[q * 8 + 4], x[q * 8 + 5]);
      w.w = ElemTraits<T>::pack2(x[q * 8 + 6], x[q * 8 + 7]);
      *reinterpret_cast<uint4*>(buf + sw64(row & 31, q)) = w;
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (ew.lane == 0) {
      tma_store_2d(map_x16, buf, n, row0);
      bulk_commit();
    }
    ew.cur ^= 1;
  }
  return ss;
}

template <typename T>
__device__ __forceinline__ void epilogue_residual(const GemmArgs& args, const CUtensorMap* map_res,
                                                  const CUtensorMap* map_x16, const TileInfo& ti, EpiWarp& ew,
                                                  uint32_t taddr, int half, int quarter, int row, long long R,
                                                  bool valid, int row0, int parity, float* red) {
  const float ss = residual_blocks<T>(args, map_res, map_x16, ti.n0, ew, taddr, half, row, valid, row0);
  float* slot = red + (parity * 2 + half) * 128;
  slot[row] = ss;
  named_barrier(1 + quarter, 64);
  if (half == 0 && valid) {
    const float total = slot[row] + red[(parity * 2 + 1) * 128 + row];
    if (args.row_sumsq_out != nullptr)
      atomicAdd(args.row_sumsq_out + R, total);   // this tile's 256 columns of a wider row
    else
      args.row_inv_out[R] = 16.0f / sqrtf(total + 1.0e-12f);   // sqrtf(256) / sqrtf(sum + 1e-12)
  }
}

// ---------------------------------------------------------------- GEGLU
// Accumulator columns interleave (value i, gate i) rows of the FFN input
// projection, so this warp's 128 columns give 64 outputs
// h = (v inv + b_v) * gelu(g inv + b_g), staged as one 32-row x 64-column block
// and written by one TMA store at output column (n0 + 128 half) / 2.
template <typename T>
__device__ __forceinline__ void epilogue_geglu(const GemmArgs& args, const CUtensorMap* map_out, const TileInfo& ti,
                                               EpiWarp& ew, uint32_t taddr, int half, int row, int row0, float inv) {
  const float2 inv2 = make_float2(inv, inv);
  uint8_t* buf = ew.buf[ew.cur];
  if (ew.lane == 0) bulk_wait_read1();   // the store that last used this buffer has read it
  __syncwarp();
#pragma unroll
  for (int hh = 0; hh < 4; ++hh) {
    const int c = half * 128 + 32 * hh;
    uint32_t r[32];
    tmem_ld32(taddr + c, r);
    tmem_wait_ld();
    reg_fence(r);
    const float4* bias = reinterpret_cast<const float4*>(args.bias + ti.n0 + c);
    float h[16];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = __ldg(bias + q);   // (value, gate, value, gate)
      const float2 val = __ffma2_rn(make_float2(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 2])), inv2,
                                    make_float2(b.x, b.z));
      const float2 gate = __ffma2_rn(make_float2(__uint_as_float(r[4 * q + 1]), __uint_as_float(r[4 * q + 3])),
                                     inv2, make_float2(b.y, b.w));
      const float2 act = __fmul2_rn(val, gelu_pair(gate));
      h[2 * q] = act.x;
      h[2 * q + 1] = act.y;
    }
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      uint4 w;
      w.x = ElemTraits<T>::pack2(h[q * 8 + 0], h[q * 8 + 1]);
      w.y = ElemTraits<T>::pack2(h[q * 8 + 2], h[q * 8 + 3]);
      w.z = ElemTraits<T>::pack2(h[q * 8 + 4], h[q * 8 + 5]);
      w.w = ElemTraits<T>::pack2(h[q * 8 + 6], h[q * 8 + 7]);
      *reinterpret_cast<uint4*>(buf + sw128(row & 31, 2 * hh + q)) = w;
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (ew.lane == 0) {
    tma_store_2d(map_out, buf, (ti.n0 + half * 128) >> 1, row0);
    bulk_commit();
  }
  ew.cur ^= 1;
}

// ---------------------------------------------------------------- direct per-row epilogues
// Grouped mask layers, the QKV gate tile and the fp32 test store.
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_direct(const GemmArgs& args, const TileInfo& ti, uint32_t taddr, int half,
                                                long long R, bool valid, float inv) {
  const int c_end = min(ti.n_size, half * 128 + 128);
  for (int c = half * 128; c < c_end; c += 32) {
    float v[32];
    int count;
    if (ti.n_size - c >= 32) {
      uint32_t r[32];
      tmem_ld32(taddr + c, r);
      tmem_wait_ld();
      reg_fence(r);
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      count = 32;
    } else {
      uint32_t r[16];
      tmem_ld16(taddr + c, r);
      tmem_wait_ld();
      reg_fence(r);
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
#pragma unroll
      for (int j = 16; j < 32; ++j) v[j] = 0.f;
      count = 16;
    }
    if (!valid) continue;
    const int n = ti.n0 + c;
    if (EPI == kEpiQkvRope) {
      // Gate tile: columns 0..7 are the 8 head-gate logits of the normed row
      // (gates :853, sigmoid in apply_gates :808-818).
      float4 g0, g1;
      g0.x = sigmoidf(v[0] * inv + __ldg(args.gate_b + 0));
      g0.y = sigmoidf(v[1] * inv + __ldg(args.gate_b + 1));
      g0.z = sigmoidf(v[2] * inv + __ldg(args.gate_b + 2));
      g0.w = sigmoidf(v[3] * inv + __ldg(args.gate_b + 3));
      g1.x = sigmoidf(v[4] * inv + __ldg(args.gate_b + 4));
      g1.y = sigmoidf(v[5] * inv + __ldg(args.gate_b + 5));
      g1.z = sigmoidf(v[6] * inv + __ldg(args.gate_b + 6));
      g1.w = sigmoidf(v[7] * inv + __ldg(args.gate_b + 7));
      reinterpret_cast<float4*>(args.gates_out + R * kHeads)[0] = g0;
      reinterpret_cast<float4*>(args.gates_out + R * kHeads)[1] = g1;
    } else if (EPI == kEpiTanhBand) {
      const float* bias = args.bias + ti.b_row + c;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = tanhf(v[j] * inv + __ldg(bias + j));
      store_row16<T>(static_cast<T*>(args.out) + R * args.ldo + n, v, count);
    } else if (EPI == kEpiStoreF32) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(args.out) + R * args.ldo + n);
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q * 4 < count) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else if (EPI == kEpiGluMask) {
      // Columns hold interleaved (value, gate) pairs of band `ti.band`; pair p
      // is mask component p of the band: frequency first + p/4, channel
      // (p/2)%2, re/im p%2 (mask_band, vocalarc_separation.c:1330-1338).
      const int band = ti.band;
      const int dim = args.band_dim != nullptr ? __ldg(args.band_dim + band) : c_band_dim[band];
      const int first = args.band_first != nullptr ? __ldg(args.band_first + band) : c_band_first[band];
      const long long seq = R / args.frames;
      const int t = static_cast<int>(R - seq * args.frames);
      const long long chunk = seq / (args.bands > 0 ? args.bands : kBands);
      const float* bias = args.bias + ti.b_row + c;
      const int p0 = n >> 1;
      if (args.mask_ref_layout) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int p = p0 + j;
          if (2 * j < count && p < dim) {
            const float value = v[2 * j] + __ldg(bias + 2 * j);
            const float gate = v[2 * j + 1] + __ldg(bias + 2 * j + 1);
            const int f = first + (p >> 2), ch = (p >> 1) & 1, ri = p & 1;
            float* dst = static_cast<float*>(args.out) +
                         ((static_cast<long long>(f) * kChannels + ch) * args.frames + t) * 2 + ri;
            *dst = value * sigmoidf(gate);
          }
        }
      } else {
        float* dst = static_cast<float*>(args.out) + ((chunk * args.frames + t) * kFreqBins + first) * 4 + p0;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int p = p0 + j;
          if (2 * j < count && p < dim) {
            const float value = v[2 * j] + __ldg(bias + 2 * j);
            const float gate = v[2 * j + 1] + __ldg(bias + 2 * j + 1);
            dst[j] = value * sigmoidf(gate);
          }
        }
      }
    }
  }
}

__device__ __forceinline__ bool wait_no_abort_check(uint64_t* bar, uint32_t parity, int* err) {
  // Bounded wait used while unwinding: ignores the abort flag.
  const unsigned long long start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicCAS(err, 0, kErrWaitDrain);
      return false;
    }
  }
  return true;
}

template <typename T, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_c, const __grid_constant__ CUtensorMap map_d,
                const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint8_t* sEpi = sB + kStages * kBBytes;
  float* red = reinterpret_cast<float*>(sEpi + kEpiWarps * 2 * kStageBuf);
  uint64_t* full = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + kRedBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint64_t* ep_bar = drain + 1;   // [8 warps][2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ep_bar + 2 * kEpiWarps);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&ep_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&map_a);
    tma_prefetch(&map_b);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < args.num_tiles && !*abort_flag; tile += gridDim.x) {
        const TileInfo ti = decode_tile(args, tile);
        const uint32_t b_bytes = args.b_box16 ? static_cast<uint32_t>(ti.n_size) * 128u : uint32_t(kBBytes);
        bool ok = true;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, args.err, kErrWaitTma)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], kABytes + b_bytes);
          tma_load_2d(sA + stage * kABytes, &map_a, &full[stage], kb * kBK, ti.a_row);
          if (args.b_box16) {
            for (int r = 0; r < ti.n_size; r += 16)
              tma_load_2d(sB + stage * kBBytes + r * 128, &map_b, &full[stage], kb * kBK, ti.b_row + r);
          } else {
            tma_load_2d(sB + stage * kBBytes, &map_b, &full[stage], kb * kBK, ti.b_row);
          }
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer: warp-uniform loop, one elected lane issues;
    // descriptors advance by constant offsets (K step of 16 = 32 bytes).
    const uint32_t idesc_base = idesc_f16(kBM, 0, ElemTraits<T>::kBf16, 0, 0);
    const uint64_t a_desc0 = sw128_desc(smem_u32(sA), 16, 1024);
    const uint64_t b_desc0 = sw128_desc(smem_u32(sB), 16, 1024);
    int stage = 0;
    uint32_t phase = 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++it) {
      const TileInfo ti = decode_tile(args, tile);
      const int acc = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
      if (!mbar_wait_warp(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.err, kErrWaitMma)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
      const uint32_t idesc = idesc_base | ((static_cast<uint32_t>(ti.n_size) >> 3) << 17);
      bool ok = true;
      for (int kb = 0; kb < args.k_blocks; ++kb) {
        if (!mbar_wait_warp(&full[stage], phase, abort_flag, args.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (elect_one()) {
          const uint64_t da = a_desc0 + static_cast<uint64_t>((stage * kABytes) >> 4);
          const uint64_t db = b_desc0 + static_cast<uint64_t>((stage * kBBytes) >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) umma_f16(d_tmem, da + 2 * kk, db + 2 * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(&acc_full[acc]);
      __syncwarp();
    }
    // Drain: every MMA issued above has completed before TMEM is released.
    if (elect_one()) {
      umma_commit(drain);
      wait_no_abort_check(drain, 0, args.err);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps 2..9: lane quarter warp%4, column half
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int ew_index = warp - 2;
    EpiWarp ew;
    ew.buf[0] = sEpi + ew_index * 2 * kStageBuf;
    ew.buf[1] = ew.buf[0] + kStageBuf;
    ew.bar[0] = &ep_bar[ew_index * 2];
    ew.bar[1] = &ep_bar[ew_index * 2 + 1];
    ew.phase[0] = ew.phase[1] = 0;
    ew.cur = 0;
    ew.lane = lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
      // Row values that do not depend on the accumulator are loaded before
      // the wait, while the tile's MMAs run.
      const TileInfo ti = decode_tile(args, tile);
      const long long R = static_cast<long long>(ti.a_row) + row;
      const bool valid = row < ti.m_valid;
      const float inv = (EPI != kEpiResidual && args.row_inv != nullptr && valid) ? __ldg(args.row_inv + R) : 1.0f;
      float4 rope[16];
      if (EPI == kEpiQkvRope) {
        const bool do_rope = valid && ti.n_size == kBN && ti.n0 < args.rope_cols;
        const int pos = static_cast<int>((R / args.pos_div) % args.pos_mod);
        const float4* table = args.rope + pos;
#pragma unroll
        for (int i = 0; i < 16; ++i)
          rope[i] = do_rope ? __ldg(table + static_cast<long long>(i) * args.rope_stride) : make_float4(1.f, 0.f, 1.f, 0.f);
      }
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, args.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);
      const int row0 = ti.a_row + quarter * 32;
      if (EPI == kEpiResidual) {
        epilogue_residual<T>(args, &map_c, &map_d, ti, ew, taddr, half, quarter, row, R, valid, row0, it & 1, red);
      } else if (EPI == kEpiGeglu) {
        epilogue_geglu<T>(args, &map_c, ti, ew, taddr, half, row, row0, inv);
      } else if ((EPI == kEpiStore || EPI == kEpiGelu || EPI == kEpiQkvRope) && ti.n_size == kBN) {
        epilogue_out16<T, EPI>(args, &map_c, ti, ew, taddr, half, row, row0, inv, rope);
      } else {
        epilogue_direct<T, EPI>(args, ti, taddr, half, R, valid, inv);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if (lane == 0) bulk_wait_all();   // outstanding tensor stores complete before exit
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- fused FFN
// x += GELU(inv * x16 W1^T + b1) W2^T + b2 for a 128-row tile, the hidden
// activations kept on chip (transformer_forward's FFN, vocalarc_separation.c:
// 866-873, with the RMSNorm gamma folded into W1).  Per tile:
//   * the tile's x16 (128 x 256, four K-blocks) stays in shared memory while
//     all hidden slices are computed;
//   * the hidden units run in slices of 128: FF1(s) accumulates into one of two
//     128-column TMEM buffers, the eight epilogue warps apply the row scale,
//     b1 and GELU and write the 16-bit slice into one of two shared-memory
//     buffers in the 128B-swizzled K-major layout of an MMA operand, and FF2(s)
//     accumulates that slice times W2[:, slice] into the 256-column output
//     accumulator;
//   * the MMA warp issues FF1(0), FF1(1), FF2(0), FF1(2), FF2(1), ... so the
//     tensor cores run FF1(s+1) and FF2(s-1) while GELU(s) is computed;
//   * W1 and W2 stream through one ring of 32 KB stages (two 128 x 64 W1
//     K-blocks, or one 256 x 64 W2 K-block) in the MMA's order;
//   * the output tile goes through the residual epilogue of the plain GEMM,
//     staged in the two hidden buffers, which are free once FF2 of the last
//     slice has completed.
// HBM traffic per row: x16 in, x in and out, x16 out (3 KB) instead of the
// 7 KB of an FF1 launch writing the hidden and an FF2 launch reading it.
namespace ffn {
constexpr int kSliceN = 128;
constexpr int kXBytes = 4 * kABytes;   // 64 KB
constexpr int kHBytes = 2 * kABytes;   // 32 KB
constexpr int kWStage = 32768;
constexpr int kWStages = 3;
constexpr int kRed = 2 * 128 * 4;      // one column half's row sums, two tile parities
constexpr int kBarCount = 40;
constexpr int kSmemBytes = 1024 + kXBytes + 2 * kHBytes + kWStages * kWStage + kRed + kBarBytes;
static_assert(kSmemBytes <= 232448, "fused FFN shared memory");
static_assert(kEpiWarps * 2 * kStageBuf == 2 * kHBytes, "residual staging is the two hidden buffers");
static_assert(kBarCount * 8 + 8 <= kBarBytes, "barrier block");
}  // namespace ffn

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    ffn_kernel(const __grid_constant__ CUtensorMap map_x16, const __grid_constant__ CUtensorMap map_w1,
               const __grid_constant__ CUtensorMap map_w2, const __grid_constant__ CUtensorMap map_res,
               const __grid_constant__ CUtensorMap map_out16, const GemmArgs args, const int slices) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sX = smem;
  uint8_t* sH = sX + ffn::kXBytes;   // [2][kHBytes]; the residual staging at the tile's end
  uint8_t* sW = sH + 2 * ffn::kHBytes;
  float* red = reinterpret_cast<float*>(sW + ffn::kWStages * ffn::kWStage);
  uint64_t* bars = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + ffn::kRed);
  uint64_t* x_full = bars + 0;
  uint64_t* x_free = bars + 1;
  uint64_t* w_full = bars + 2;       // [3]
  uint64_t* w_empty = bars + 5;      // [3]
  uint64_t* acc1_full = bars + 8;    // [2]
  uint64_t* acc1_empty = bars + 10;  // [2]
  uint64_t* h_full = bars + 12;      // [2]
  uint64_t* h_free = bars + 14;      // [2]
  uint64_t* acc2_full = bars + 16;
  uint64_t* acc2_empty = bars + 17;
  uint64_t* stage_free = bars + 18;
  uint64_t* red_full = bars + 19;    // [4]
  uint64_t* drain = bars + 23;
  uint64_t* ep_bar = bars + 24;      // [8 warps][2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + ffn::kBarCount);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  if (threadIdx.x == 0) {
    mbar_init(x_full, 1);
    mbar_init(x_free, 1);
    for (int s = 0; s < ffn::kWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc1_full[b], 1);
      mbar_init(&acc1_empty[b], kEpiWarps);
      mbar_init(&h_full[b], kEpiWarps);
      mbar_init(&h_free[b], 1);
    }
    mbar_init(acc2_full, 1);
    mbar_init(acc2_empty, kEpiWarps);
    mbar_init(stage_free, kEpiWarps);
    for (int q = 0; q < 4; ++q) mbar_init(&red_full[q], 32);
    mbar_init(drain, 1);
    for (int i = 0; i < 2 * kEpiWarps; ++i) mbar_init(&ep_bar[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch(&map_x16);
    tma_prefetch(&map_w1);
    tma_prefetch(&map_w2);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer: x16 per tile, then W1 / W2 stages in the MMA's order.
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_phase[ffn::kWStages] = {0, 0, 0};
      bool used[ffn::kWStages] = {false, false, false};
      int x_loads = 0;
      bool ok = true;
      auto next_stage = [&]() -> bool {
        if (!mbar_wait(&w_empty[stage], phase ^ 1u, abort_flag, args.err, kErrWaitTma)) return false;
        mbar_arrive_expect_tx(&w_full[stage], ffn::kWStage);
        used[stage] = true;
        last_phase[stage] = phase;
        return true;
      };
      auto advance = [&]() {
        if (++stage == ffn::kWStages) {
          stage = 0;
          phase ^= 1u;
        }
      };
      auto load_w1 = [&](int s) -> bool {
        for (int j = 0; j < 2; ++j) {
          if (!next_stage()) return false;
          uint8_t* dst = sW + stage * ffn::kWStage;
          tma_load_2d(dst, &map_w1, &w_full[stage], (2 * j) * kBK, s * ffn::kSliceN);
          tma_load_2d(dst + kABytes, &map_w1, &w_full[stage], (2 * j + 1) * kBK, s * ffn::kSliceN);
          advance();
        }
        return true;
      };
      auto load_w2 = [&](int s) -> bool {
        for (int j = 0; j < 2; ++j) {
          if (!next_stage()) return false;
          tma_load_2d(sW + stage * ffn::kWStage, &map_w2, &w_full[stage], s * ffn::kSliceN + j * kBK, 0);
          advance();
        }
        return true;
      };
      int it = 0;
      for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x, ++it) {
        const int a_row = tile * kBM;
        if (!mbar_wait(x_free, (static_cast<uint32_t>(it) & 1u) ^ 1u, abort_flag, args.err, kErrWaitTma)) break;
        mbar_arrive_expect_tx(x_full, ffn::kXBytes);
        for (int kb = 0; kb < 4; ++kb) tma_load_2d(sX + kb * kABytes, &map_x16, x_full, kb * kBK, a_row);
        ++x_loads;
        // The tile's fp32 residual rows (contiguous, 1 KB each) into L2 for the epilogue.
        const int rows = min(kBM, args.m_rows - a_row);
        prefetch_l2_bulk(static_cast<const float*>(args.out) + static_cast<long long>(a_row) * 256,
                         static_cast<uint32_t>(rows) * 1024u);
        ok = load_w1(0) && (slices < 2 || load_w1(1));
        for (int s = 0; s < slices && ok; ++s) ok = load_w2(s) && (s + 2 >= slices || load_w1(s + 2));
      }
      // Every load issued has landed before the CTA can exit.
      if (x_loads > 0) wait_no_abort_check(x_full, static_cast<uint32_t>(x_loads - 1) & 1u, args.err);
      for (int s = 0; s < ffn::kWStages; ++s)
        if (used[s]) wait_no_abort_check(&w_full[s], last_phase[s], args.err);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (one elected lane of a converged warp)
    const uint32_t idesc1 = idesc_f16(kBM, ffn::kSliceN, ElemTraits<T>::kBf16, 0, 0);
    const uint32_t idesc2 = idesc_f16(kBM, kBN, ElemTraits<T>::kBf16, 0, 0);
    const uint64_t x_desc0 = sw128_desc(smem_u32(sX), 16, 1024);
    const uint64_t h_desc0 = sw128_desc(smem_u32(sH), 16, 1024);
    const uint64_t w_desc0 = sw128_desc(smem_u32(sW), 16, 1024);
    int stage = 0;
    uint32_t phase = 0;
    int g1 = 0, g2 = 0;   // FF1 / FF2 slices issued so far
    auto wait_stage = [&]() -> bool {
      if (!mbar_wait_warp(&w_full[stage], phase, abort_flag, args.err, kErrWaitMma)) return false;
      tc_fence_after();
      return true;
    };
    auto advance = [&]() {
      if (++stage == ffn::kWStages) {
        stage = 0;
        phase ^= 1u;
      }
    };
    auto issue_ff1 = [&]() -> bool {
      const int b = g1 & 1;
      if (!mbar_wait_warp(&acc1_empty[b], (static_cast<uint32_t>(g1 >> 1) & 1u) ^ 1u, abort_flag, args.err,
                          kErrWaitMma))
        return false;
      tc_fence_after();
      const uint32_t d = tmem_base + static_cast<uint32_t>(kBN + ffn::kSliceN * b);
      for (int j = 0; j < 2; ++j) {
        if (!wait_stage()) return false;
        if (elect_one()) {
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint64_t da = x_desc0 + static_cast<uint64_t>(((2 * j + i) * kABytes) >> 4);
            const uint64_t db = w_desc0 + static_cast<uint64_t>((stage * ffn::kWStage + i * kABytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              umma_f16(d, da + 2 * kk, db + 2 * kk, idesc1, (j | i | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&w_empty[stage]);
        }
        __syncwarp();
        advance();
      }
      if (elect_one()) umma_commit(&acc1_full[b]);
      __syncwarp();
      ++g1;
      return true;
    };
    auto issue_ff2 = [&](int s) -> bool {
      const int b = g2 & 1;
      if (!mbar_wait_warp(&h_full[b], static_cast<uint32_t>(g2 >> 1) & 1u, abort_flag, args.err, kErrWaitMma))
        return false;
      tc_fence_after();
      for (int j = 0; j < 2; ++j) {
        if (!wait_stage()) return false;
        if (elect_one()) {
          const uint64_t da = h_desc0 + static_cast<uint64_t>((b * ffn::kHBytes + j * kABytes) >> 4);
          const uint64_t db = w_desc0 + static_cast<uint64_t>((stage * ffn::kWStage) >> 4);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            umma_f16(tmem_base, da + 2 * kk, db + 2 * kk, idesc2, (s | j | kk) != 0 ? 1u : 0u);
          umma_commit(&w_empty[stage]);
        }
        __syncwarp();
        advance();
      }
      if (elect_one()) umma_commit(&h_free[b]);
      __syncwarp();
      ++g2;
      return true;
    };
    auto release_x = [&]() {
      if (elect_one()) umma_commit(x_free);
      __syncwarp();
    };
    int it = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++it) {
      if (!mbar_wait_warp(x_full, static_cast<uint32_t>(it) & 1u, abort_flag, args.err, kErrWaitMma)) break;
      tc_fence_after();
      bool ok = issue_ff1() && (slices < 2 || issue_ff1());
      if (ok && slices <= 2) release_x();
      // FF2(0) overwrites the output accumulator: the previous tile's epilogue has read it.
      ok = ok && mbar_wait_warp(acc2_empty, (static_cast<uint32_t>(it) & 1u) ^ 1u, abort_flag, args.err, kErrWaitMma);
      if (ok) tc_fence_after();
      for (int s = 0; s < slices && ok; ++s) {
        ok = issue_ff2(s);
        if (ok && s + 2 < slices) {
          ok = issue_ff1();
          if (ok && s + 2 == slices - 1) release_x();
        }
      }
      if (!ok) break;
      if (elect_one()) umma_commit(acc2_full);
      __syncwarp();
    }
    if (elect_one()) {
      umma_commit(drain);
      wait_no_abort_check(drain, 0, args.err);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps 2..9: lane quarter warp % 4, column half
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    const int ew_index = warp - 2;
    EpiWarp ew;
    ew.buf[0] = sH + ew_index * 2 * kStageBuf;
    ew.buf[1] = ew.buf[0] + kStageBuf;
    ew.bar[0] = &ep_bar[ew_index * 2];
    ew.bar[1] = &ep_bar[ew_index * 2 + 1];
    ew.phase[0] = ew.phase[1] = 0;
    ew.cur = 0;
    ew.lane = lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    int g = 0;
    int it = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++it) {
      const int a_row = tile * kBM;
      const long long R = static_cast<long long>(a_row) + row;
      const bool valid = row < args.m_rows - a_row;
      // A plain load: this kernel rewrites the same rows' factor at the tile's end.
      const float inv = valid ? args.row_inv[R] : 1.0f;
      const float2 inv2 = make_float2(inv, inv);
      bool ok = true;
      for (int s = 0; s < slices; ++s, ++g) {
        const int b = g & 1;
        const uint32_t gp = static_cast<uint32_t>(g >> 1) & 1u;
        if (!mbar_wait_warp(&acc1_full[b], gp, abort_flag, args.err, kErrWaitEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[2][32];
        const uint32_t taddr = lane_base + static_cast<uint32_t>(kBN + ffn::kSliceN * b + 64 * half);
        tmem_ld32(taddr, r[0]);
        tmem_ld32(taddr + 32, r[1]);
        tmem_wait_ld();
        reg_fence(r[0]);
        reg_fence(r[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc1_empty[b]);
        // The hidden buffer is free once FF2 of slice g - 2 has read it, and
        // at a tile's first slice once the previous tile's output stores have
        // read the staging.
        if (!mbar_wait_warp(&h_free[b], gp ^ 1u, abort_flag, args.err, kErrWaitEpilogue) ||
            (s == 0 && !mbar_wait_warp(stage_free, (static_cast<uint32_t>(it) & 1u) ^ 1u, abort_flag, args.err,
                                       kErrWaitEpilogue))) {
          ok = false;
          break;
        }
        uint8_t* dst = sH + b * ffn::kHBytes + half * kABytes;
        const float* b1 = args.bias1 + s * ffn::kSliceN + 64 * half;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          float v[32];
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float4 bv = __ldg(reinterpret_cast<const float4*>(b1 + 32 * hh) + q);
            const float2 lo = __ffma2_rn(make_float2(__uint_as_float(r[hh][4 * q]), __uint_as_float(r[hh][4 * q + 1])),
                                         inv2, make_float2(bv.x, bv.y));
            const float2 hi = __ffma2_rn(
                make_float2(__uint_as_float(r[hh][4 * q + 2]), __uint_as_float(r[hh][4 * q + 3])), inv2,
                make_float2(bv.z, bv.w));
            const float2 g0 = gelu_pair(lo);
            const float2 g1 = gelu_pair(hi);
            v[4 * q] = g0.x;
            v[4 * q + 1] = g0.y;
            v[4 * q + 2] = g1.x;
            v[4 * q + 3] = g1.y;
          }
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = ElemTraits<T>::pack2(v[q * 8 + 0], v[q * 8 + 1]);
            w.y = ElemTraits<T>::pack2(v[q * 8 + 2], v[q * 8 + 3]);
            w.z = ElemTraits<T>::pack2(v[q * 8 + 4], v[q * 8 + 5]);
            w.w = ElemTraits<T>::pack2(v[q * 8 + 6], v[q * 8 + 7]);
            *reinterpret_cast<uint4*>(dst + sw128(row, 4 * hh + q)) = w;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[b]);
      }
      if (!ok) break;
      if (!mbar_wait_warp(acc2_full, static_cast<uint32_t>(it) & 1u, abort_flag, args.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const float ss = residual_blocks<T>(args, &map_res, &map_out16, 0, ew, lane_base, half, row, valid,
                                          a_row + quarter * 32);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc2_empty);
      // inv of the new row from both column halves' sums of squares.
      float* slot = red + (it & 1) * 128;
      if (half == 1) {
        slot[row] = ss;
        mbar_arrive(&red_full[quarter]);
      } else {
        if (!mbar_wait_warp(&red_full[quarter], static_cast<uint32_t>(it) & 1u, abort_flag, args.err,
                            kErrWaitEpilogue))
          break;
        if (valid) args.row_inv_out[R] = 16.0f / sqrtf(ss + slot[row] + 1.0e-12f);   // sqrtf(256) / sqrtf(sum + 1e-12)
      }
      // This warp's output stores have read the staging (part of the hidden buffers).
      if (lane == 0) {
        bulk_wait_read0();
        mbar_arrive(stage_free);
      }
      __syncwarp();
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <typename T, int EPI>
cudaError_t launch_typed(const GemmMaps& maps, const GemmArgs& args, int sm_count, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  const cudaError_t e = opt_in_smem(gemm_kernel<T, EPI>, kSmemBytes, configured);
  if (e != cudaSuccess) return e;
  if (args.num_tiles <= 0) return cudaSuccess;
  const int grid = args.num_tiles < sm_count ? args.num_tiles : sm_count;
  gemm_kernel<T, EPI><<<grid, kThreads, kSmemBytes, stream>>>(maps.a, maps.b, maps.c, maps.d, args);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch(int epilogue, const GemmMaps& m, const GemmArgs& args, int sms, cudaStream_t s) {
  switch (epilogue) {
    case kEpiStore: return launch_typed<T, kEpiStore>(m, args, sms, s);
    case kEpiGelu: return launch_typed<T, kEpiGelu>(m, args, sms, s);
    case kEpiQkvRope: return launch_typed<T, kEpiQkvRope>(m, args, sms, s);
    case kEpiResidual: return launch_typed<T, kEpiResidual>(m, args, sms, s);
    case kEpiTanhBand: return launch_typed<T, kEpiTanhBand>(m, args, sms, s);
    case kEpiGluMask: return launch_typed<T, kEpiGluMask>(m, args, sms, s);
    case kEpiStoreF32: return launch_typed<T, kEpiStoreF32>(m, args, sms, s);
    case kEpiGeglu: return launch_typed<T, kEpiGeglu>(m, args, sms, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_gemm(int epilogue, bool bf16, const GemmMaps& maps, const GemmArgs& args, int sm_count,
                        cudaStream_t stream) {
  return bf16 ? dispatch<__nv_bfloat16>(epilogue, maps, args, sm_count, stream)
              : dispatch<__half>(epilogue, maps, args, sm_count, stream);
}

cudaError_t launch_ffn(bool bf16, const FfnMaps& maps, const GemmArgs& args, int hidden, int sm_count,
                       cudaStream_t stream) {
  if (hidden <= 0 || hidden % ffn::kSliceN != 0) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> configured_h{0}, configured_b{0};
  const cudaError_t e = bf16 ? opt_in_smem(ffn_kernel<__nv_bfloat16>, ffn::kSmemBytes, configured_b)
                             : opt_in_smem(ffn_kernel<__half>, ffn::kSmemBytes, configured_h);
  if (e != cudaSuccess) return e;
  if (args.num_tiles <= 0) return cudaSuccess;
  const int grid = args.num_tiles < sm_count ? args.num_tiles : sm_count;
  const int slices = hidden / ffn::kSliceN;
  if (bf16)
    ffn_kernel<__nv_bfloat16><<<grid, kThreads, ffn::kSmemBytes, stream>>>(maps.x16, maps.w1, maps.w2, maps.res,
                                                                           maps.out16, args, slices);
  else
    ffn_kernel<__half><<<grid, kThreads, ffn::kSmemBytes, stream>>>(maps.x16, maps.w1, maps.w2, maps.res, maps.out16,
                                                                   args, slices);
  return cudaGetLastError();
}

cudaError_t upload_band_tables(const int* first, const int* dims) {
  cudaError_t e = cudaMemcpyToSymbol(c_band_first, first, sizeof(int) * kBands);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(c_band_dim, dims, sizeof(int) * kBands);
}

}  // namespace vab
