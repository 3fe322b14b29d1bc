// Persistent tcgen05 GEMM for sm_100a:  C[M][N] = A[M][K] * B[N][K]^T.
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
// (coefficients fitted here, minimax in h; x is clamped there, where h is
// within 3.4e-6 of 0 or 1): |h error| <= 1.9e-5 with an exact tanh.  tanh runs
// on MUFU (tanh.approx.f32; measured on the B200: relative error below
// 2^-16.6), so a value costs one MUFU operation and seven FMA-pipe operations
// instead of the sixteen of a polynomial for erf itself, which made the FFN
// input GEMM's epilogue FMA-bound.  Measured GELU error: max 5.5e-5, rms
// 2.4e-5 absolute -- below the 16-bit rounding of the stored hidden value.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float2 gelu_pair(float2 x) {
  const float2 xc = make_float2(fminf(fmaxf(x.x, -4.5f), 4.5f), fminf(fmaxf(x.y, -4.5f), 4.5f));
  const float2 x2 = __fmul2_rn(xc, xc);
  float2 p = __ffma2_rn(x2, make_float2(-0.00031580726499669254f, -0.00031580726499669254f),
                        make_float2(0.03679825738072395f, 0.03679825738072395f));
  p = __ffma2_rn(p, x2, make_float2(0.797717809677124f, 0.797717809677124f));
  const float2 g = __fmul2_rn(p, xc);
  const float2 h = __ffma2_rn(make_float2(tanh_approx(g.x), tanh_approx(g.y)), make_float2(0.5f, 0.5f),
                              make_float2(0.5f, 0.5f));
  return __fmul2_rn(x, h);
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
template <typename T>
__device__ __forceinline__ void epilogue_residual(const GemmArgs& args, const CUtensorMap* map_res,
                                                  const CUtensorMap* map_x16, const TileInfo& ti, EpiWarp& ew,
                                                  uint32_t taddr, int half, int quarter, int row, long long R,
                                                  bool valid, int row0, int parity, float* red) {
  float ss = 0.f;
  // Prefetch the first residual block of this warp's columns.
  if (ew.lane == 0) {
    bulk_wait_read0();
    mbar_arrive_expect_tx(ew.bar[ew.cur], kStageBuf);
    tma_load_2d(ew.buf[ew.cur], map_res, ew.bar[ew.cur], ti.n0 + half * 128, row0);
  }
  __syncwarp();
#pragma unroll 1
  for (int s = 0; s < 4; ++s) {
    const int b = ew.cur;
    const int c = half * 128 + s * 32;
    const int n = ti.n0 + c;
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
        const float4* table = reinterpret_cast<const float4*>(args.rope + static_cast<long long>(pos) * (kDimHead / 2));
#pragma unroll
        for (int i = 0; i < 16; ++i) rope[i] = do_rope ? __ldg(table + i) : make_float4(1.f, 0.f, 1.f, 0.f);
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

cudaError_t upload_band_tables(const int* first, const int* dims) {
  cudaError_t e = cudaMemcpyToSymbol(c_band_first, first, sizeof(int) * kBands);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(c_band_dim, dims, sizeof(int) * kBands);
}

}  // namespace vab
