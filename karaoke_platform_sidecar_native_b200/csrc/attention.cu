// tcgen05 flash attention for the axial RoPE transformer (sm_100a).
//
// One CTA computes 128 queries of one (sequence, head): softmax(Q K^T / 8) V,
// non-causal, head dim 64, then multiplies by the per-head sigmoid gate.  It
// replaces the reference's one-warp-per-query SIMT kernel (time axis,
// native/native_gpu_cuda.cu:299-331) and its pack / two cuBLAS batched GEMMs /
// softmax / reorder chain (band axis, :339-401, :497-538); the CPU semantics
// are attention_heads + apply_gates (native/vocalarc_separation.c:753-818).
//
// Warp 0: TMA loads of Q (once) and K/V tiles through a 4-D tensor map that
// addresses the token layout directly (no pack or transpose kernels).
// Warp 1: one thread issues S = Q K^T (M=128, N<=128, K=64) into TMEM and
// O_j = P_j V_j (M=128, N=64, K<=128, V as an MN-major operand).
// Warps 2-5: one thread per query row; read S from TMEM, online softmax in
// fp32 with exp2, write P (16-bit) to 128-byte-swizzled shared memory, and
// accumulate the per-tile O_j from TMEM in registers with the rescale factor.
#include "ptx.cuh"
#include "vab_internal.h"

namespace vab {

namespace {

constexpr int kThreads = 192;
constexpr int kTile = 128;
constexpr int kQBytes = kTile * kDimHead * 2;   // 16 KB
constexpr int kPBytes = kTile * kTile * 2;      // 32 KB
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;

template <int NBUF>
struct AttnSmem {
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;
  static constexpr int kV = kK + NBUF * kQBytes;
  static constexpr int kP = kV + NBUF * kQBytes;
  static constexpr int kBar = kP + NBUF * kPBytes;
  static constexpr int kBytes = 1024 + kBar + 256;
  static constexpr uint32_t kTmemCols = NBUF == 2 ? 512u : 256u;
};

__device__ __forceinline__ int round16(int x) { return (x + 15) & ~15; }

__device__ __forceinline__ bool wait_drain(uint64_t* bar, uint32_t parity, int* err) {
  const unsigned long long start = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - start > kWaitLimitNs) {
      atomicCAS(err, 0, kErrWaitDrain);
      return false;
    }
  }
  return true;
}

template <typename T, int NBUF>
__global__ void __launch_bounds__(kThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map, const AttnArgs args) {
  using L = AttnSmem<NBUF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sP = smem + L::kP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + NBUF;
  uint64_t* s_full = kv_empty + NBUF;
  uint64_t* s_empty = s_full + NBUF;
  uint64_t* p_full = s_empty + NBUF;
  uint64_t* o_full = p_full + NBUF;
  uint64_t* o_empty = o_full + NBUF;
  uint64_t* drain = o_empty + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();

  // Work item: (query tile, head, sequence), query tile fastest so that CTAs
  // sharing K/V run together and hit L2.
  const long long bid = blockIdx.x;
  const int q_tile = static_cast<int>(bid % args.q_tiles);
  const long long rest = bid / args.q_tiles;
  const int head = static_cast<int>(rest % kHeads);
  const long long seq = rest / kHeads;
  const int q0 = q_tile * kTile;
  const int length = args.length;
  const int nkv = (length + kTile - 1) / kTile;
  int c_a, c_b;  // the two non-position coordinates of the tensor map
  if (args.pos_dim == 1) {
    c_a = static_cast<int>(seq % args.d2);
    c_b = static_cast<int>(seq / args.d2);
  } else {
    c_a = static_cast<int>(seq % args.d1);
    c_b = static_cast<int>(seq / args.d1);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, L::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint32_t tmem_s = tmem_base;                       // NBUF x 128 columns
  const uint32_t tmem_o = tmem_base + NBUF * kTile;        // NBUF x 64 columns

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&map);
      auto load_tile = [&](uint8_t* dst, uint64_t* bar, int col, int pos) {
        if (args.pos_dim == 1)
          tma_load_4d(dst, &map, bar, col, pos, c_a, c_b);
        else
          tma_load_4d(dst, &map, bar, col, c_a, pos, c_b);
      };
      mbar_arrive_expect_tx(q_full, kQBytes);
      load_tile(sQ, q_full, head * kDimHead, q0);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % NBUF;
        const uint32_t par = static_cast<uint32_t>(j / NBUF) & 1u;
        if (!mbar_wait(&kv_empty[st], par ^ 1u, abort_flag, args.err, kErrWaitTma)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kQBytes);
        load_tile(sK + st * kQBytes, &kv_full[st], kDimInner + head * kDimHead, j * kTile);
        load_tile(sV + st * kQBytes, &kv_full[st], 2 * kDimInner + head * kDimHead, j * kTile);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t bf = ElemTraits<T>::kBf16;
      const uint32_t q_addr = smem_u32(sQ);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % NBUF;
        const uint32_t par = static_cast<uint32_t>(i / NBUF) & 1u;
        if (!mbar_wait(&p_full[st], par, abort_flag, args.err, kErrWaitMma)) return false;
        if (!mbar_wait(&o_empty[st], par ^ 1u, abort_flag, args.err, kErrWaitMma)) return false;
        tc_fence_after();
        const int nc = min(kTile, round16(length - i * kTile));
        const uint32_t idesc = idesc_f16(kTile, kDimHead, bf, 0, 1);
        const uint32_t p_addr = smem_u32(sP + st * kPBytes);
        const uint32_t v_addr = smem_u32(sV + st * kQBytes);
        for (int kk = 0; kk < nc / 16; ++kk) {
          const uint64_t da = sw128_desc(p_addr + (kk >> 2) * (kTile * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t db = sw128_desc(v_addr + kk * 2048, 8192, 1024);
          umma_f16(tmem_o + st * kDimHead, da, db, idesc, kk != 0 ? 1u : 0u);
        }
        umma_commit(&o_full[st]);
        umma_commit(&kv_empty[st]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, args.err, kErrWaitMma);
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % NBUF;
        const uint32_t par = static_cast<uint32_t>(j / NBUF) & 1u;
        if (!mbar_wait(&kv_full[st], par, abort_flag, args.err, kErrWaitMma)) { ok = false; break; }
        if (!mbar_wait(&s_empty[st], par ^ 1u, abort_flag, args.err, kErrWaitMma)) { ok = false; break; }
        tc_fence_after();
        const int nc = min(kTile, round16(length - j * kTile));
        const uint32_t idesc = idesc_f16(kTile, static_cast<uint32_t>(nc), bf, 0, 0);
        const uint32_t k_addr = smem_u32(sK + st * kQBytes);
#pragma unroll
        for (int kk = 0; kk < kDimHead / 16; ++kk) {
          const uint64_t da = sw128_desc(q_addr + kk * 32, 16, 1024);
          const uint64_t db = sw128_desc(k_addr + kk * 32, 16, 1024);
          umma_f16(tmem_s + st * kTile, da, db, idesc, kk != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        if (j > 0 && !issue_pv(j - 1)) { ok = false; break; }
      }
      if (ok) issue_pv(nkv - 1);
      umma_commit(drain);
      wait_drain(drain, 0, args.err);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / correction / epilogue warps
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    float o_acc[kDimHead];
#pragma unroll
    for (int d = 0; d < kDimHead; ++d) o_acc[d] = 0.f;
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 0.f;
    bool ok = true;

    auto accumulate_o = [&](int i, float alpha) -> bool {
      const int st = i % NBUF;
      const uint32_t par = static_cast<uint32_t>(i / NBUF) & 1u;
      if (!mbar_wait_warp(&o_full[st], par, abort_flag, args.err, kErrWaitSoftmax)) return false;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32(tmem_o + st * kDimHead + lane_off, r0);
      tmem_ld32(tmem_o + st * kDimHead + 32 + lane_off, r1);
      tmem_wait_ld();
      reg_fence(r0);
      reg_fence(r1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[st]);
#pragma unroll
      for (int d = 0; d < 32; ++d) {
        o_acc[d] = o_acc[d] * alpha + __uint_as_float(r0[d]);
        o_acc[32 + d] = o_acc[32 + d] * alpha + __uint_as_float(r1[d]);
      }
      return true;
    };

    for (int j = 0; j < nkv; ++j) {
      const int st = j % NBUF;
      const uint32_t par = static_cast<uint32_t>(j / NBUF) & 1u;
      if (!mbar_wait_warp(&s_full[st], par, abort_flag, args.err, kErrWaitSoftmax)) { ok = false; break; }
      tc_fence_after();
      const int kv0 = j * kTile;
      const int valid = length - kv0;
      const int nc = min(kTile, round16(valid));
      const uint32_t s_addr = tmem_s + st * kTile + lane_off;
      // Pass 1: row maximum over the valid keys.
      float mx = -INFINITY;
      for (int c = 0; c < nc; c += 32) {
        float v[32];
        if (nc - c >= 32) {
          uint32_t r[32];
          tmem_ld32(s_addr + c, r);
          tmem_wait_ld();
          reg_fence(r);
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]);
        } else {
          uint32_t r[16];
          tmem_ld16(s_addr + c, r);
          tmem_wait_ld();
          reg_fence(r);
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = __uint_as_float(r[q]);
#pragma unroll
          for (int q = 16; q < 32; ++q) v[q] = -INFINITY;
        }
#pragma unroll
        for (int q = 0; q < 32; ++q) mx = fmaxf(mx, (c + q < valid) ? v[q] : -INFINITY);
      }
      const float m_new = fmaxf(m_run, mx);
      const float alpha = ex2_approx((m_run - m_new) * kScaleLog2);
      const float mscaled = m_new * kScaleLog2;
      // Pass 2: probabilities, row sum, P tile (16-bit) into swizzled smem.
      float sum = 0.f;
      uint8_t* p_base = sP + st * kPBytes + (row >> 3) * 1024 + (row & 7) * 128;
      for (int c = 0; c < nc; c += 32) {
        float v[32];
        const int cnt = (nc - c >= 32) ? 32 : 16;
        if (cnt == 32) {
          uint32_t r[32];
          tmem_ld32(s_addr + c, r);
          tmem_wait_ld();
          reg_fence(r);
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = __uint_as_float(r[q]);
        } else {
          uint32_t r[16];
          tmem_ld16(s_addr + c, r);
          tmem_wait_ld();
          reg_fence(r);
#pragma unroll
          for (int q = 0; q < 16; ++q) v[q] = __uint_as_float(r[q]);
#pragma unroll
          for (int q = 16; q < 32; ++q) v[q] = 0.f;
        }
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const float p = (c + q < valid) ? ex2_approx(fmaf(v[q], kScaleLog2, -mscaled)) : 0.f;
          v[q] = p;
          sum += p;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          if (g * 8 < cnt) {
            const int key = c + g * 8;
            const int atom = key >> 6;
            const int chunk16 = (key & 63) >> 3;
            uint4 w;
            w.x = ElemTraits<T>::pack2(v[g * 8 + 0], v[g * 8 + 1]);
            w.y = ElemTraits<T>::pack2(v[g * 8 + 2], v[g * 8 + 3]);
            w.z = ElemTraits<T>::pack2(v[g * 8 + 4], v[g * 8 + 5]);
            w.w = ElemTraits<T>::pack2(v[g * 8 + 6], v[g * 8 + 7]);
            *reinterpret_cast<uint4*>(p_base + atom * (kTile * 128) + ((chunk16 ^ (row & 7)) << 4)) = w;
          }
        }
      }
      tc_fence_before();
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s_empty[st]);
        mbar_arrive(&p_full[st]);
      }
      l_run = l_run * alpha + sum;
      if (j > 0 && !accumulate_o(j - 1, alpha_prev)) { ok = false; break; }
      alpha_prev = alpha;
      m_run = m_new;
    }
    if (ok) ok = accumulate_o(nkv - 1, alpha_prev);
    const int qpos = q0 + row;
    if (ok && qpos < length) {
      long long R;
      if (args.pos_dim == 1)
        R = seq * args.d1 + qpos;
      else
        R = (static_cast<long long>(c_b) * args.d2 + qpos) * args.d1 + c_a;
      const float scale = __ldg(args.gates + R * kHeads + head) / l_run;
      uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(args.out) + R * kDimInner + head * kDimHead);
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        uint4 w;
        w.x = ElemTraits<T>::pack2(o_acc[g * 8 + 0] * scale, o_acc[g * 8 + 1] * scale);
        w.y = ElemTraits<T>::pack2(o_acc[g * 8 + 2] * scale, o_acc[g * 8 + 3] * scale);
        w.z = ElemTraits<T>::pack2(o_acc[g * 8 + 4] * scale, o_acc[g * 8 + 5] * scale);
        w.w = ElemTraits<T>::pack2(o_acc[g * 8 + 6] * scale, o_acc[g * 8 + 7] * scale);
        dst[g] = w;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

template <typename T, int NBUF>
cudaError_t launch_typed(const CUtensorMap& map, const AttnArgs& args, cudaStream_t stream) {
  using L = AttnSmem<NBUF>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel<T, NBUF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::kBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const long long blocks = static_cast<long long>(args.q_tiles) * kHeads * args.sequences;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  attention_kernel<T, NBUF><<<static_cast<unsigned>(blocks), kThreads, L::kBytes, stream>>>(map, args);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Long sequences (L > 128): one CTA computes two 128-query tiles (A, B) of one
// (sequence, head) that share every K/V tile.  Warps 2-5 own tile A, warps 6-9
// tile B (one query row per thread).  O accumulates in TMEM across KV tiles;
// a row's reference maximum m is raised only when a tile's maximum exceeds it
// by more than 2^8 in exp2 units, in which case that row of O (TMEM) and its
// running sum are rescaled -- otherwise P = exp2((s - m) c) <= 256 stays exact
// enough in 16 bits and no O traffic is needed.
constexpr int kPairThreads = 320;
constexpr float kRescaleLog2 = 8.0f;

constexpr int kKvStages = 3;   // K/V ring depth: loads run two tiles ahead of the PV that frees a stage

struct PairSmem {
  static constexpr int kQ = 0;                       // 2 x 16 KB
  static constexpr int kK = kQ + 2 * kQBytes;        // kKvStages x 16 KB
  static constexpr int kV = kK + kKvStages * kQBytes;  // kKvStages x 16 KB
  static constexpr int kP = kV + kKvStages * kQBytes;  // 2 tiles x 32 KB
  static constexpr int kBar = kP + 2 * kPBytes;
  static constexpr int kBytes = 1024 + kBar + 256;
};

template <typename T>
__global__ void __launch_bounds__(kPairThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap map, const AttnArgs args) {
  using L = PairSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sP = smem + L::kP;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;                 // [kKvStages]
  uint64_t* kv_empty = kv_full + kKvStages;     // [kKvStages]
  uint64_t* s_full = kv_empty + kKvStages;      // [tile]
  uint64_t* s_empty = s_full + 2;               // [tile]
  uint64_t* p_full = s_empty + 2;               // [tile]
  uint64_t* o_full = p_full + 2;                // [tile]
  uint64_t* drain = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const long long bid = blockIdx.x;
  const int q_pairs = (args.q_tiles + 1) / 2;
  const int pair = static_cast<int>(bid % q_pairs);
  const long long rest = bid / q_pairs;
  const int head = static_cast<int>(rest % kHeads);
  const long long seq = rest / kHeads;
  const int q0 = pair * 2 * kTile;
  const int length = args.length;
  const int ntiles = (q0 + kTile < length) ? 2 : 1;
  const int nkv = (length + kTile - 1) / kTile;
  int c_a, c_b;
  if (args.pos_dim == 1) {
    c_a = static_cast<int>(seq % args.d2);
    c_b = static_cast<int>(seq / args.d2);
  } else {
    c_a = static_cast<int>(seq % args.d1);
    c_b = static_cast<int>(seq / args.d1);
  }

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // TMEM columns: S_A [0,128), S_B [128,256), O_A [256,320), O_B [320,384).

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&map);
      auto load_tile = [&](uint8_t* dst, uint64_t* bar, int col, int pos) {
        if (args.pos_dim == 1)
          tma_load_4d(dst, &map, bar, col, pos, c_a, c_b);
        else
          tma_load_4d(dst, &map, bar, col, c_a, pos, c_b);
      };
      mbar_arrive_expect_tx(q_full, ntiles * kQBytes);
      load_tile(sQ, q_full, head * kDimHead, q0);
      if (ntiles == 2) load_tile(sQ + kQBytes, q_full, head * kDimHead, q0 + kTile);
      for (int j = 0; j < nkv; ++j) {
        const int st = j % kKvStages;
        const uint32_t par = static_cast<uint32_t>(j / kKvStages) & 1u;
        if (!mbar_wait(&kv_empty[st], par ^ 1u, abort_flag, args.err, kErrWaitTma)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * kQBytes);
        load_tile(sK + st * kQBytes, &kv_full[st], kDimInner + head * kDimHead, j * kTile);
        load_tile(sV + st * kQBytes, &kv_full[st], 2 * kDimInner + head * kDimHead, j * kTile);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t bf = ElemTraits<T>::kBf16;
      auto issue_pv = [&](int i) -> bool {
        const int st = i % kKvStages;
        const int nc = min(kTile, round16(length - i * kTile));
        const uint32_t idesc = idesc_f16(kTile, kDimHead, bf, 0, 1);
        const uint32_t v_addr = smem_u32(sV + st * kQBytes);
        for (int x = 0; x < ntiles; ++x) {
          if (!mbar_wait(&p_full[x], static_cast<uint32_t>(i) & 1u, abort_flag, args.err, kErrWaitMma)) return false;
          tc_fence_after();
          const uint32_t p_addr = smem_u32(sP + x * kPBytes);
          for (int kk = 0; kk < nc / 16; ++kk) {
            const uint64_t da = sw128_desc(p_addr + (kk >> 2) * (kTile * 128) + (kk & 3) * 32, 16, 1024);
            const uint64_t db = sw128_desc(v_addr + kk * 2048, 8192, 1024);
            umma_f16(tmem_base + 256 + x * kDimHead, da, db, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&o_full[x]);
        }
        umma_commit(&kv_empty[st]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, args.err, kErrWaitMma);
      for (int j = 0; ok && j < nkv; ++j) {
        const int st = j % kKvStages;
        if (!mbar_wait(&kv_full[st], static_cast<uint32_t>(j / kKvStages) & 1u, abort_flag, args.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        const int nc = min(kTile, round16(length - j * kTile));
        const uint32_t idesc = idesc_f16(kTile, static_cast<uint32_t>(nc), bf, 0, 0);
        const uint32_t k_addr = smem_u32(sK + st * kQBytes);
        for (int x = 0; x < ntiles && ok; ++x) {
          if (!mbar_wait(&s_empty[x], (static_cast<uint32_t>(j) & 1u) ^ 1u, abort_flag, args.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + x * kQBytes);
#pragma unroll
          for (int kk = 0; kk < kDimHead / 16; ++kk) {
            const uint64_t da = sw128_desc(q_addr + kk * 32, 16, 1024);
            const uint64_t db = sw128_desc(k_addr + kk * 32, 16, 1024);
            umma_f16(tmem_base + x * kTile, da, db, idesc, kk != 0 ? 1u : 0u);
          }
          umma_commit(&s_full[x]);
        }
        if (ok && j > 0 && !issue_pv(j - 1)) ok = false;
      }
      if (ok) issue_pv(nkv - 1);
      umma_commit(drain);
      wait_drain(drain, 0, args.err);
    }
    __syncwarp();
  } else {
    const int x = (warp - 2) >> 2;          // query tile of this warp
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem_base + x * kTile + lane_off;
    const uint32_t o_addr = tmem_base + 256 + x * kDimHead + lane_off;
    uint8_t* p_base = sP + x * kPBytes + (row >> 3) * 1024 + (row & 7) * 128;
    bool ok = x < ntiles;
    float m_ref = -INFINITY;   // reference maximum (raw score units)
    float l_run = 0.f;
    for (int j = 0; ok && j < nkv; ++j) {
      if (!mbar_wait_warp(&s_full[x], static_cast<uint32_t>(j) & 1u, abort_flag, args.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int valid = length - j * kTile;
      const int nc = min(kTile, round16(valid));
      // The tile is processed as two 64-column halves.  The reference maximum
      // only has to keep exp2 below 2^8, so each half is exponentiated against
      // the current reference; when the second half raises it, the packed P of
      // the first half is rescaled.  All 128 S columns are read; columns >=
      // valid (stale, or never written by a narrower MMA) are masked.
      uint32_t pk[kTile / 2];   // P packed to 16-bit pairs
      float sum = 0.f;
      float factor = 1.0f;      // accumulated rescale of O and l for this tile
      bool raised = false;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t ra[32], rb[32];
        tmem_ld32(s_addr + 64 * hh, ra);
        tmem_ld32(s_addr + 64 * hh + 32, rb);
        tmem_wait_ld();
        reg_fence(ra);
        reg_fence(rb);
        if (hh == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s_empty[x]);   // S buffer free for the next tile
        }
        float v[64];
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          v[q] = __uint_as_float(ra[q]);
          v[32 + q] = __uint_as_float(rb[q]);
        }
        if (valid < kTile) {   // only the last KV tile has keys past the end
#pragma unroll
          for (int q = 0; q < 64; ++q)
            if (64 * hh + q >= valid) v[q] = -INFINITY;
        }
        float mxs[8];
#pragma unroll
        for (int a = 0; a < 8; ++a) mxs[a] = v[a];
#pragma unroll
        for (int q = 8; q < 64; ++q) mxs[q & 7] = fmaxf(mxs[q & 7], v[q]);
        const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                               fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
        // Raise the reference maximum only when this half would exceed 2^8.
        if ((mx - m_ref) * kScaleLog2 > kRescaleLog2) {
          const float f = ex2_approx((m_ref - mx) * kScaleLog2);   // 0 when m_ref = -inf
          m_ref = mx;
          factor *= f;
          sum *= f;
          raised = true;
          if (hh == 1) {
            const uint32_t f2 = ElemTraits<T>::pack2(f, f);
#pragma unroll
            for (int q = 0; q < 32; ++q) pk[q] = ElemTraits<T>::mul2(pk[q], f2);
          }
        }
        const float mscaled = m_ref * kScaleLog2;
        float sums[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int q = 0; q < 64; q += 2) {
          const float p0 = ex2_approx(fmaf(v[q], kScaleLog2, -mscaled));
          const float p1 = ex2_approx(fmaf(v[q + 1], kScaleLog2, -mscaled));
          sums[(q >> 1) & 7] += p0 + p1;
          pk[32 * hh + q / 2] = ElemTraits<T>::pack2(p0, p1);
        }
        sum += ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]));
      }
      const bool raise = raised;
      if (j > 0) {
        // PV of the previous tile must be complete before P is overwritten and
        // before this row of O is rescaled.
        if (!mbar_wait_warp(&o_full[x], static_cast<uint32_t>(j - 1) & 1u, abort_flag, args.err, kErrWaitSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t r[32];
            tmem_ld32(o_addr + half * 32, r);
            tmem_wait_ld();
            reg_fence(r);
#pragma unroll
            for (int d = 0; d < 32; ++d) r[d] = __float_as_uint(__uint_as_float(r[d]) * factor);
            tmem_st32(o_addr + half * 32, r);
          }
          tmem_wait_st();
        }
      }
      l_run = l_run * factor + sum;
#pragma unroll
      for (int g = 0; g < kTile / 8; ++g) {
        if (g * 8 < nc) {
          const int atom = g >> 3;
          const int chunk16 = g & 7;
          *reinterpret_cast<uint4*>(p_base + atom * (kTile * 128) + ((chunk16 ^ (row & 7)) << 4)) =
              make_uint4(pk[g * 4 + 0], pk[g * 4 + 1], pk[g * 4 + 2], pk[g * 4 + 3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[x]);
    }
    if (ok && mbar_wait_warp(&o_full[x], static_cast<uint32_t>(nkv - 1) & 1u, abort_flag, args.err, kErrWaitSoftmax)) {
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32(o_addr, r0);
      tmem_ld32(o_addr + 32, r1);
      tmem_wait_ld();
      reg_fence(r0);
      reg_fence(r1);
      const int qpos = q0 + x * kTile + row;
      if (qpos < length) {
        long long R;
        if (args.pos_dim == 1)
          R = seq * args.d1 + qpos;
        else
          R = (static_cast<long long>(c_b) * args.d2 + qpos) * args.d1 + c_a;
        const float scale = __ldg(args.gates + R * kHeads + head) / l_run;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(args.out) + R * kDimInner + head * kDimHead);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 w;
          w.x = ElemTraits<T>::pack2(__uint_as_float(r0[g * 8 + 0]) * scale, __uint_as_float(r0[g * 8 + 1]) * scale);
          w.y = ElemTraits<T>::pack2(__uint_as_float(r0[g * 8 + 2]) * scale, __uint_as_float(r0[g * 8 + 3]) * scale);
          w.z = ElemTraits<T>::pack2(__uint_as_float(r0[g * 8 + 4]) * scale, __uint_as_float(r0[g * 8 + 5]) * scale);
          w.w = ElemTraits<T>::pack2(__uint_as_float(r0[g * 8 + 6]) * scale, __uint_as_float(r0[g * 8 + 7]) * scale);
          dst[g] = w;
        }
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 w;
          w.x = ElemTraits<T>::pack2(__uint_as_float(r1[g * 8 + 0]) * scale, __uint_as_float(r1[g * 8 + 1]) * scale);
          w.y = ElemTraits<T>::pack2(__uint_as_float(r1[g * 8 + 2]) * scale, __uint_as_float(r1[g * 8 + 3]) * scale);
          w.z = ElemTraits<T>::pack2(__uint_as_float(r1[g * 8 + 4]) * scale, __uint_as_float(r1[g * 8 + 5]) * scale);
          w.w = ElemTraits<T>::pack2(__uint_as_float(r1[g * 8 + 6]) * scale, __uint_as_float(r1[g * 8 + 7]) * scale);
          dst[4 + g] = w;
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <typename T>
cudaError_t launch_pair(const CUtensorMap& map, const AttnArgs& args, cudaStream_t stream) {
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(attention_pair_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         PairSmem::kBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const long long blocks = static_cast<long long>((args.q_tiles + 1) / 2) * kHeads * args.sequences;
  if (blocks <= 0) return cudaSuccess;
  if (blocks > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  attention_pair_kernel<T><<<static_cast<unsigned>(blocks), kPairThreads, PairSmem::kBytes, stream>>>(map, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_attention(bool bf16, const CUtensorMap& map_qkv, const AttnArgs& args, cudaStream_t stream) {
  // Single-tile sequences (band axis, L <= 128) use one buffer of each kind:
  // 80 KB of shared memory and 256 TMEM columns, two CTAs per SM.  Longer
  // sequences use the two-query-tile kernel.
  const bool single = args.length <= kTile;
  if (bf16)
    return single ? launch_typed<__nv_bfloat16, 1>(map_qkv, args, stream) : launch_pair<__nv_bfloat16>(map_qkv, args, stream);
  return single ? launch_typed<__half, 1>(map_qkv, args, stream) : launch_pair<__half>(map_qkv, args, stream);
}

}  // namespace vab
