// Persistent tcgen05 GEMM for sm_100a:  C[M][N] = A[M][K] * B[N][K]^T.
//
// One CTA per SM walks a static tile schedule.  Warp 0 issues TMA loads of
// 128x64 A and (n_size)x64 B tiles into a 4-stage 128-byte-swizzled ring, warp
// 1 (one thread) issues tcgen05.mma (M=128, N=n_size<=256, K=16) into one of
// two TMEM accumulators, and warps 2-9 (two per TMEM lane quarter, splitting
// the columns) drain the other accumulator with tcgen05.ld and apply a fused
// epilogue (RoPE, bias+GELU, fp32 residual, tanh,
// GLU + complex-mask scatter).  The reference computes these products with
// cuBLAS SGEMM plus separate SIMT kernels (native/native_gpu_cuda.cu:540-552,
// :279-297, :414-426, :453-485).
#include <cstdio>

#include "ptx.cuh"
#include "vab_internal.h"

namespace vab {

namespace {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 64;
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 2;   // 16 KB
constexpr int kBBytes = kBN * kBK * 2;   // 32 KB
constexpr int kThreads = 320;          // TMA warp, MMA warp, 8 epilogue warps
constexpr int kEpiWarps = 8;
constexpr int kTmemCols = 512;           // two 128x256 fp32 accumulators
constexpr size_t kSmemBytes = 1024 + kStages * (kABytes + kBBytes) + 256;

__constant__ int c_band_first[kBands];
__constant__ int c_band_dim[kBands];

struct TileInfo {
  int a_row, b_row, n0, m_valid, n_size, band;
};

__device__ __forceinline__ TileInfo decode_tile(const GemmArgs& args, int tile) {
  TileInfo t;
  if (args.tiles == nullptr) {
    const int m_blk = tile / args.n_tiles;
    const int n_blk = tile - m_blk * args.n_tiles;
    t.a_row = m_blk * kBM;
    t.m_valid = min(kBM, args.m_rows - t.a_row);
    t.b_row = n_blk * kBN;
    t.n0 = n_blk * kBN;
    t.n_size = kBN;
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

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865475f)); }

__device__ __forceinline__ float sigmoidf(float x) { return 1.0f / (1.0f + __expf(-x)); }

template <typename T>
__device__ __forceinline__ void store_row16(T* dst, const float* v, int count) {
  // count is 16 or 32; dst is 32-byte aligned.
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

// Applies the epilogue to `count` (16 or 32) accumulator columns [c, c+count)
// of tile row `r` (global A row R).
template <typename T, int EPI>
__device__ __forceinline__ void epilogue_chunk(const GemmArgs& args, const TileInfo& ti, long long R, int c,
                                               float (&v)[32], int count, const float4 (&rope)[8]) {
  const int n = ti.n0 + c;  // output column of v[0]
  if (EPI == kEpiStore || EPI == kEpiGelu || EPI == kEpiTanhBand) {
    const float* bias = args.bias;
    const int bias_base = (EPI == kEpiTanhBand) ? (ti.b_row + c) : n;
    if (bias != nullptr) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < count) v[j] += __ldg(bias + bias_base + j);
    }
    if (EPI == kEpiGelu) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
    }
    if (EPI == kEpiTanhBand) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = tanhf(v[j]);
    }
    T* dst = static_cast<T*>(args.out) + R * args.ldo + n;
    store_row16<T>(dst, v, count);
  } else if (EPI == kEpiStoreF32) {
    float4* dst = reinterpret_cast<float4*>(static_cast<float*>(args.out) + R * args.ldo + n);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      if (q * 4 < count) dst[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else if (EPI == kEpiQkvRope) {
    // rope[i] = (cos, sin, cos, sin) of pairs 2i, 2i+1 of this 32-column chunk
    // (the chunk starts at column n, pair (n % 64) / 2, of a 64-wide head).
    if (n < args.rope_cols) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 cs = rope[i];
        float a = v[4 * i], b = v[4 * i + 1];
        v[4 * i] = a * cs.x - b * cs.y;
        v[4 * i + 1] = a * cs.y + b * cs.x;
        a = v[4 * i + 2];
        b = v[4 * i + 3];
        v[4 * i + 2] = a * cs.z - b * cs.w;
        v[4 * i + 3] = a * cs.w + b * cs.z;
      }
    }
    T* dst = static_cast<T*>(args.out) + R * args.ldo + n;
    store_row16<T>(dst, v, count);
  } else if (EPI == kEpiResidual) {
    float4* dst = reinterpret_cast<float4*>(args.resid + R * args.ldr + n);
    const float* bias = args.bias;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q * 4 < count) {
        float4 x = dst[q];
        float b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
        if (bias != nullptr) {
          b0 = __ldg(bias + n + 4 * q);
          b1 = __ldg(bias + n + 4 * q + 1);
          b2 = __ldg(bias + n + 4 * q + 2);
          b3 = __ldg(bias + n + 4 * q + 3);
        }
        x.x += v[4 * q] + b0;
        x.y += v[4 * q + 1] + b1;
        x.z += v[4 * q + 2] + b2;
        x.w += v[4 * q + 3] + b3;
        dst[q] = x;
      }
    }
  } else if (EPI == kEpiGluMask) {
    // Columns hold interleaved (value, gate) pairs of band `ti.band`; pair p
    // is mask component p of the band: frequency first + p/4, channel
    // (p/2)%2, re/im p%2 (mask_band, vocalarc_separation.c:1330-1338).
    const int band = ti.band;
    const int dim = c_band_dim[band];
    const int first = c_band_first[band];
    const long long seq = R / args.frames;
    const int t = static_cast<int>(R - seq * args.frames);
    const long long chunk = seq / kBands;
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
      float* dst = static_cast<float*>(args.out) +
                   ((chunk * args.frames + t) * kFreqBins + first) * 4 + p0;
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
                const GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sB + kStages * kBBytes);
  uint64_t* empty = full + kStages;
  uint64_t* acc_full = empty + kStages;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
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
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t idesc_base = idesc_f16(kBM, 0, ElemTraits<T>::kBf16, 0, 0);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      for (int tile = blockIdx.x; tile < args.num_tiles && !*abort_flag; tile += gridDim.x, ++it) {
        const TileInfo ti = decode_tile(args, tile);
        const int acc = it & 1;
        const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, args.err, kErrWaitMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * kBN);
        const uint32_t idesc = idesc_base | ((static_cast<uint32_t>(ti.n_size) >> 3) << 17);
        bool ok = true;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, args.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * kABytes);
          const uint32_t b_base = smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t da = sw128_desc(a_base + kk * 32, 16, 1024);
            const uint64_t db = sw128_desc(b_base + kk * 32, 16, 1024);
            umma_f16(d_tmem, da, db, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
      }
      // Drain: every MMA issued above has completed before TMEM is released.
      umma_commit(drain);
      wait_no_abort_check(drain, 0, args.err);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue warps 2..9: lane quarter warp%4, column half
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row = quarter * 32 + lane;
    int it = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = static_cast<uint32_t>(it >> 1) & 1u;
      if (!mbar_wait_warp(&acc_full[acc], acc_phase, abort_flag, args.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const TileInfo ti = decode_tile(args, tile);
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>(acc * kBN);
      const long long R = static_cast<long long>(ti.a_row) + row;
      const bool valid = row < ti.m_valid;
      // A 32-column chunk of this half always starts at column 32*half of a
      // 64-wide head, so it uses RoPE pairs [16*half, 16*half + 16) of the
      // row's position: load them once per tile.
      float4 rope[8];
      if (EPI == kEpiQkvRope) {
        const int pos = static_cast<int>((R / args.pos_div) % args.pos_mod);
        const float4* table = reinterpret_cast<const float4*>(args.rope + static_cast<long long>(pos) * (kDimHead / 2) + 16 * half);
#pragma unroll
        for (int i = 0; i < 8; ++i) rope[i] = valid && ti.n0 < args.rope_cols ? __ldg(table + i) : make_float4(1.f, 0.f, 1.f, 0.f);
      }
      for (int c = half * 32; c < ti.n_size; c += 64) {
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
        if (valid) epilogue_chunk<T, EPI>(args, ti, R, c, v, count, rope);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <typename T, int EPI>
cudaError_t launch_typed(const CUtensorMap& map_a, const CUtensorMap& map_b, const GemmArgs& args,
                         int sm_count, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel<T, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if (args.num_tiles <= 0) return cudaSuccess;
  const int grid = args.num_tiles < sm_count ? args.num_tiles : sm_count;
  gemm_kernel<T, EPI><<<grid, kThreads, kSmemBytes, stream>>>(map_a, map_b, args);
  return cudaGetLastError();
}

template <typename T>
cudaError_t dispatch(int epilogue, const CUtensorMap& a, const CUtensorMap& b, const GemmArgs& args, int sms,
                     cudaStream_t s) {
  switch (epilogue) {
    case kEpiStore: return launch_typed<T, kEpiStore>(a, b, args, sms, s);
    case kEpiGelu: return launch_typed<T, kEpiGelu>(a, b, args, sms, s);
    case kEpiQkvRope: return launch_typed<T, kEpiQkvRope>(a, b, args, sms, s);
    case kEpiResidual: return launch_typed<T, kEpiResidual>(a, b, args, sms, s);
    case kEpiTanhBand: return launch_typed<T, kEpiTanhBand>(a, b, args, sms, s);
    case kEpiGluMask: return launch_typed<T, kEpiGluMask>(a, b, args, sms, s);
    case kEpiStoreF32: return launch_typed<T, kEpiStoreF32>(a, b, args, sms, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_gemm(int epilogue, bool bf16, const CUtensorMap& map_a, const CUtensorMap& map_b,
                        const GemmArgs& args, int sm_count, cudaStream_t stream) {
  return bf16 ? dispatch<__nv_bfloat16>(epilogue, map_a, map_b, args, sm_count, stream)
              : dispatch<__half>(epilogue, map_a, map_b, args, sm_count, stream);
}

cudaError_t upload_band_tables(const int* first, const int* dims) {
  cudaError_t e = cudaMemcpyToSymbol(c_band_first, first, sizeof(int) * kBands);
  if (e != cudaSuccess) return e;
  return cudaMemcpyToSymbol(c_band_dim, dims, sizeof(int) * kBands);
}

}  // namespace vab
