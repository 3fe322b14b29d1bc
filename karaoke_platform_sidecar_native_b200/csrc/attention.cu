// tcgen05 flash attention for the axial RoPE transformer (sm_100a).
//
// softmax(Q K^T / 8) V per (sequence, head), non-causal, head dim 64, then
// multiplied by the per-head sigmoid gate.  It
// replaces the reference's one-warp-per-query SIMT kernel (time axis,
// native/native_gpu_cuda.cu:299-331) and its pack / two cuBLAS batched GEMMs /
// softmax / reorder chain (band axis, :339-401, :497-538); the CPU semantics
// are attention_heads + apply_gates (native/vocalarc_separation.c:753-818).
//
// Both kernels below share one structure.  Warp 0 issues TMA loads of Q, K, V
// through a 4-D tensor map that addresses the token layout directly (no pack
// or transpose kernels).  Warp 1 (one thread) issues S = Q K^T (M=128,
// N<=128, K=64) into TMEM and O = P V (M=128, N=64, K<=128, V as an MN-major
// operand).  Warps 2-9, one thread per query row, read S from TMEM, compute
// the softmax in fp32 with exp2 and write P (16-bit) to 128-byte-swizzled
// shared memory.
#include "ptx.cuh"
#include "vab_internal.h"

namespace vab {

namespace {

constexpr int kTile = 128;
constexpr int kQBytes = kTile * kDimHead * 2;   // 16 KB
constexpr int kPBytes = kTile * kTile * 2;      // 32 KB
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;

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


// 2^x on the FMA pipe for a pair of values, x <= 8 (x < -125 is clamped; the
// result is then below 2^-124 and rounds to zero in 16 bits).  x = j + f with
// j = rint(x) from the 1.5 * 2^23 addition, f in [-1/2, 1/2]; 2^f from a
// degree-3 polynomial (coefficients fitted here for minimum relative error on
// [-1/2, 1/2], max relative error 7.5e-5, below 16-bit rounding); 2^j is added
// to the exponent field.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kMagic = 12582912.0f;
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(kMagic, kMagic));
  const float2 j = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), x);
  float2 p = __ffma2_rn(f, make_float2(0.05517097935080528f, 0.05517097935080528f),
                        make_float2(0.24260970950126648f, 0.24260970950126648f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999281764030457f, 0.9999281764030457f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Of every 8 exponent pairs, this many go to the FMA-pipe polynomial and the
// rest to MUFU ex2 (16 results per clock per SM), balancing the two pipes;
// 2 of 8 measured fastest against 0, 3 and 4.
constexpr int kPolyPairs = 2;
// The band-axis kernel is paced by its per-item latency, not by MUFU: all its
// exponentials go to MUFU (0 of 8 measured 0.564 ms against 0.588, 0.71 and
// 0.72 ms for 2, 1 and 3 of 8 on 4 chunks at L = 90).
constexpr int kItemPolyPairs = 0;

// ---------------------------------------------------------------------------
// Long sequences (L > 128): a persistent CTA walks units of two 128-query
// tiles (A, B) of one (sequence, head), which share every K/V tile.  Warps 2-5
// own tile A, warps 6-9 tile B (one query row per thread).  Barrier phases
// and the K/V ring run on across units and Q is double-buffered, so the next
// unit's Q load and first S overlap this unit's last tiles and output.  P goes
// to tensor memory and the PV MMA reads it from there (A operand in TMEM), so
// P never touches shared memory.  O accumulates in TMEM across KV tiles; a
// row's reference maximum m is raised only when a tile's maximum exceeds it by
// more than 2^8 in exp2 units, in which case that row of O (TMEM) and its
// running sum are rescaled -- otherwise P = exp2((s - m) c) <= 256 stays exact
// enough in 16 bits and no O traffic is needed.
//
// Two issuer warps run warp-uniform loops and issue each MMA under
// elect.sync, with descriptors advanced by constant offsets: warp 1 issues
// S = Q K^T as soon as a tile's S buffer is free, warp 10 issues O += P V as
// soon as a tile's P is in TMEM, so neither waits behind the other's
// dependencies; each commits its reads of a K/V stage to kv_empty (count 2).
constexpr int kPairThreads = 352;   // warps: TMA, S issuer, 8 softmax, PV issuer
constexpr float kRescaleLog2 = 8.0f;

constexpr int kKvStages = 3;   // K/V ring depth: loads run two tiles ahead of the PV that frees a stage

struct PairSmem {
  static constexpr int kQ = 0;                         // 2 buffers x 2 tiles x 16 KB
  static constexpr int kK = kQ + 4 * kQBytes;          // kKvStages x 16 KB
  static constexpr int kV = kK + kKvStages * kQBytes;  // kKvStages x 16 KB
  static constexpr int kBar = kV + kKvStages * kQBytes;
  static constexpr int kBytes = 1024 + kBar + 256;
};

// TMEM columns: S_A [0,128), S_B [128,256), O_A [256,320), O_B [320,384),
// P_A [384,448), P_B [448,512) (P: two 16-bit values per column).
constexpr uint32_t kColS = 0, kColO = 256, kColP = 384;

// One unit of the pair kernel: two query tiles of one (sequence, head).
struct PairUnit {
  int q0, ntiles, head, c_a, c_b;
  long long seq;
};

__device__ __forceinline__ PairUnit pair_unit(const AttnArgs& args, long long u) {
  const int q_pairs = (args.q_tiles + 1) / 2;
  PairUnit p;
  const int pair = static_cast<int>(u % q_pairs);
  const long long rest = u / q_pairs;
  p.head = static_cast<int>(rest % kHeads);
  p.seq = rest / kHeads;
  p.q0 = pair * 2 * kTile;
  p.ntiles = (p.q0 + kTile < args.length) ? 2 : 1;
  if (args.pos_dim == 1) {
    p.c_a = static_cast<int>(p.seq % args.d2);
    p.c_b = static_cast<int>(p.seq / args.d2);
  } else {
    p.c_a = static_cast<int>(p.seq % args.d1);
    p.c_b = static_cast<int>(p.seq / args.d1);
  }
  return p;
}

template <typename T>
__global__ void __launch_bounds__(kPairThreads, 1)
    attention_pair_kernel(const __grid_constant__ CUtensorMap map, const AttnArgs args, long long units) {
  using L = PairSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* q_full = bars;                      // [Q buffer]
  uint64_t* q_empty = bars + 2;                 // [Q buffer]
  uint64_t* kv_full = bars + 4;                 // [kKvStages]
  uint64_t* kv_empty = kv_full + kKvStages;     // [kKvStages]
  uint64_t* s_full = kv_empty + kKvStages;      // [tile]
  uint64_t* s_empty = s_full + 2;               // [tile]
  uint64_t* p_full = s_empty + 2;               // [tile]
  uint64_t* o_full = p_full + 2;                // [tile]
  uint64_t* o_empty = o_full + 2;               // [tile]
  uint64_t* drain = o_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int length = args.length;
  const int nkv = (length + kTile - 1) / kTile;
  const int n_local =
      static_cast<long long>(blockIdx.x) < units ? static_cast<int>((units - 1 - blockIdx.x) / gridDim.x) + 1 : 0;
  auto unit_of = [&](int lu) { return static_cast<long long>(blockIdx.x) + static_cast<long long>(lu) * gridDim.x; };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < kKvStages; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);   // S issuer (K read) and PV issuer (V read)
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(drain + 1, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch(&map);
      int kvc = 0;   // K/V tiles loaded so far (ring position)
      bool ok = true;
      for (int lu = 0; ok && lu < n_local; ++lu) {
        const PairUnit pu = pair_unit(args, unit_of(lu));
        auto load_tile = [&](uint8_t* dst, uint64_t* bar, int col, int pos) {
          if (args.pos_dim == 1)
            tma_load_4d(dst, &map, bar, col, pos, pu.c_a, pu.c_b);
          else
            tma_load_4d(dst, &map, bar, col, pu.c_a, pos, pu.c_b);
        };
        const int qb = lu & 1;
        if (!mbar_wait(&q_empty[qb], (static_cast<uint32_t>(lu >> 1) & 1u) ^ 1u, abort_flag, args.err, kErrWaitTma))
          break;
        uint8_t* q_dst = sQ + qb * 2 * kQBytes;
        mbar_arrive_expect_tx(&q_full[qb], pu.ntiles * kQBytes);
        load_tile(q_dst, &q_full[qb], pu.head * kDimHead, pu.q0);
        if (pu.ntiles == 2) load_tile(q_dst + kQBytes, &q_full[qb], pu.head * kDimHead, pu.q0 + kTile);
        for (int j = 0; j < nkv; ++j, ++kvc) {
          const int st = kvc % kKvStages;
          const uint32_t par = static_cast<uint32_t>(kvc / kKvStages) & 1u;
          if (!mbar_wait(&kv_empty[st], par ^ 1u, abort_flag, args.err, kErrWaitTma)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * kQBytes);
          load_tile(sK + st * kQBytes, &kv_full[st], kDimInner + pu.head * kDimHead, j * kTile);
          load_tile(sV + st * kQBytes, &kv_full[st], 2 * kDimInner + pu.head * kDimHead, j * kTile);
        }
      }
    }
  } else if (warp == 1) {
    // S issuer: warp-uniform, one elected lane issues S = Q K^T per tile as
    // soon as the tile's S buffer is free, independent of the PV issuer.
    const uint32_t bf = ElemTraits<T>::kBf16;
    const uint64_t q_desc = sw128_desc(smem_u32(sQ), 16, 1024);
    const uint64_t k_desc = sw128_desc(smem_u32(sK), 16, 1024);
    int sc[2] = {0, 0};   // S MMAs issued per tile
    bool ok = true;
    int kvc = 0;
    for (int lu = 0; ok && lu < n_local; ++lu) {
      const PairUnit pu = pair_unit(args, unit_of(lu));
      const int qb = lu & 1;
      if (!mbar_wait_warp(&q_full[qb], static_cast<uint32_t>(lu >> 1) & 1u, abort_flag, args.err, kErrWaitMma)) {
        ok = false;
        break;
      }
      for (int j = 0; ok && j < nkv; ++j, ++kvc) {
        const int st = kvc % kKvStages;
        if (!mbar_wait_warp(&kv_full[st], static_cast<uint32_t>(kvc / kKvStages) & 1u, abort_flag, args.err,
                            kErrWaitMma)) {
          ok = false;
          break;
        }
        const int nc = min(kTile, round16(length - j * kTile));
        const uint32_t idesc_s = idesc_f16(kTile, static_cast<uint32_t>(nc), bf, 0, 0);
        const uint64_t kd = k_desc + static_cast<uint64_t>((st * kQBytes) >> 4);
        for (int x = 0; x < pu.ntiles && ok; ++x) {
          if (!mbar_wait_warp(&s_empty[x], (static_cast<uint32_t>(sc[x]) & 1u) ^ 1u, abort_flag, args.err,
                              kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint64_t qd = q_desc + static_cast<uint64_t>(((qb * 2 + x) * kQBytes) >> 4);
#pragma unroll
            for (int kk = 0; kk < kDimHead / 16; ++kk)
              umma_f16(tmem_base + kColS + x * kTile, qd + 2 * kk, kd + 2 * kk, idesc_s, kk != 0 ? 1u : 0u);
            umma_commit(&s_full[x]);
            if (j == nkv - 1 && x == pu.ntiles - 1) umma_commit(&q_empty[qb]);   // Q buffer free after the last S
          }
          __syncwarp();
          ++sc[x];
        }
        if (ok && elect_one()) umma_commit(&kv_empty[st]);   // K of this stage read
        __syncwarp();
      }
    }
    if (elect_one()) {
      umma_commit(drain);
      wait_drain(drain, 0, args.err);
    }
    __syncwarp();
  } else if (warp == 10) {
    // PV issuer: O_x += P_x V as soon as tile x's P is in TMEM.
    const uint32_t bf = ElemTraits<T>::kBf16;
    const uint32_t idesc_o = idesc_f16(kTile, kDimHead, bf, 0, 1);
    const uint64_t v_desc = sw128_desc(smem_u32(sV), 8192, 1024);
    int pc[2] = {0, 0};   // PV MMAs issued per tile
    int uc[2] = {0, 0};   // units whose O has been completed per tile
    bool ok = true;
    int kvc = 0;
    for (int lu = 0; ok && lu < n_local; ++lu) {
      const PairUnit pu = pair_unit(args, unit_of(lu));
      for (int j = 0; ok && j < nkv; ++j, ++kvc) {
        const int st = kvc % kKvStages;
        const int ksteps = min(kTile, round16(length - j * kTile)) / 16;
        const uint64_t vd = v_desc + static_cast<uint64_t>((st * kQBytes) >> 4);
        for (int x = 0; x < pu.ntiles && ok; ++x) {
          if (!mbar_wait_warp(&p_full[x], static_cast<uint32_t>(pc[x]) & 1u, abort_flag, args.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          // The first PV of a unit overwrites O: the previous unit's O must have been read.
          if (j == 0 && uc[x] > 0 &&
              !mbar_wait_warp(&o_empty[x], static_cast<uint32_t>(uc[x] - 1) & 1u, abort_flag, args.err,
                              kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t o_col = tmem_base + kColO + x * kDimHead;
            const uint32_t p_col = tmem_base + kColP + x * (kTile / 2);
#pragma unroll
            for (int kk = 0; kk < kTile / 16; ++kk)
              if (kk < ksteps)
                umma_f16_ts(o_col, p_col + kk * 8, vd + (kk * 2048 >> 4), idesc_o, (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&o_full[x]);
          }
          __syncwarp();
          ++pc[x];
          if (j == nkv - 1) ++uc[x];
        }
        if (ok && elect_one()) umma_commit(&kv_empty[st]);   // V of this stage read
        __syncwarp();
      }
    }
    if (elect_one()) {
      umma_commit(drain + 1);
      wait_drain(drain + 1, 0, args.err);
    }
    __syncwarp();
  } else {
    const int x = (warp - 2) >> 2;          // query tile of this warp
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem_base + kColS + x * kTile + lane_off;
    const uint32_t o_addr = tmem_base + kColO + x * kDimHead + lane_off;
    const uint32_t p_addr = tmem_base + kColP + x * (kTile / 2) + lane_off;
    int c = 0;   // S tiles consumed by this tile slot so far
    bool ok = true;
    for (int lu = 0; ok && lu < n_local; ++lu) {
      const PairUnit pu = pair_unit(args, unit_of(lu));
      if (x >= pu.ntiles) continue;
      float m_ref = -INFINITY;   // reference maximum (raw score units)
      float l_run = 0.f;
      for (int j = 0; ok && j < nkv; ++j, ++c) {
        if (!mbar_wait_warp(&s_full[x], static_cast<uint32_t>(c) & 1u, abort_flag, args.err, kErrWaitSoftmax)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const int valid = length - j * kTile;
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
          for (int q = 8; q + 16 <= 64; q += 16)   // columns 8..55
#pragma unroll
            for (int a = 0; a < 8; ++a) mxs[a] = fmax3(mxs[a], v[q + a], v[q + 8 + a]);
#pragma unroll
          for (int a = 0; a < 8; ++a) mxs[a] = fmaxf(mxs[a], v[56 + a]);   // columns 56..63
          const float mx = fmax3(fmax3(mxs[0], mxs[1], mxs[2]), fmax3(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
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
          const float2 c2 = make_float2(kScaleLog2, kScaleLog2);
          const float2 nm2 = make_float2(-mscaled, -mscaled);
          float2 sums[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                            make_float2(0.f, 0.f)};
#pragma unroll
          for (int q = 0; q < 64; q += 2) {
            const float2 x2 = __ffma2_rn(make_float2(v[q], v[q + 1]), c2, nm2);
            float2 p2;
            if (((q >> 1) & 7) < kPolyPairs) {
              p2 = exp2_poly2(x2);
            } else {
              p2.x = ex2_approx(x2.x);
              p2.y = ex2_approx(x2.y);
            }
            sums[(q >> 1) & 3] = __fadd2_rn(sums[(q >> 1) & 3], p2);
            pk[32 * hh + q / 2] = ElemTraits<T>::pack2(p2.x, p2.y);
          }
          const float2 s01 = __fadd2_rn(__fadd2_rn(sums[0], sums[1]), __fadd2_rn(sums[2], sums[3]));
          sum += s01.x + s01.y;
        }
        const bool raise = raised;
        if (c > 0) {
          // PV of the previous tile must be complete before P is overwritten
          // and (within a unit) before this row of O is rescaled.
          if (!mbar_wait_warp(&o_full[x], static_cast<uint32_t>(c - 1) & 1u, abort_flag, args.err,
                              kErrWaitSoftmax)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (j > 0 && __any_sync(0xffffffffu, raise)) {
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
          }
        }
        l_run = l_run * factor + sum;
        {
          uint32_t p0[32], p1[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            p0[q] = pk[q];
            p1[q] = pk[32 + q];
          }
          tmem_st32(p_addr, p0);
          tmem_st32(p_addr + 32, p1);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      if (!ok) break;
      // Unit output: wait for the last PV, read O, release it, store.
      if (!mbar_wait_warp(&o_full[x], static_cast<uint32_t>(c - 1) & 1u, abort_flag, args.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r0[32], r1[32];
      tmem_ld32(o_addr, r0);
      tmem_ld32(o_addr + 32, r1);
      tmem_wait_ld();
      reg_fence(r0);
      reg_fence(r1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[x]);
      const int qpos = pu.q0 + x * kTile + row;
      if (qpos < length) {
        long long R;
        if (args.pos_dim == 1)
          R = pu.seq * args.d1 + qpos;
        else
          R = (static_cast<long long>(pu.c_b) * args.d2 + qpos) * args.d1 + pu.c_a;
        const float scale = __ldg(args.gates + R * kHeads + pu.head) / l_run;
        uint4* dst = reinterpret_cast<uint4*>(static_cast<T*>(args.out) + R * kDimInner + pu.head * kDimHead);
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
cudaError_t launch_pair(const CUtensorMap& map, const AttnArgs& args, int sm_count, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  const cudaError_t e = opt_in_smem(attention_pair_kernel<T>, PairSmem::kBytes, configured);
  if (e != cudaSuccess) return e;
  const long long units = static_cast<long long>((args.q_tiles + 1) / 2) * kHeads * args.sequences;
  if (units <= 0) return cudaSuccess;
  const int grid = units < sm_count ? static_cast<int>(units) : sm_count;
  attention_pair_kernel<T><<<grid, kPairThreads, PairSmem::kBytes, stream>>>(map, args, units);
  return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Short sequences (L <= 128, the band axis: L = 90): a persistent CTA walks
// (sequence, head) items.  The kernel moves about 46 KB per item (q, k, v in,
// gated output out), so the design keeps loads in flight and every stage busy:
// Q and K (freed when S = Q K^T completes) and V (freed when O = P V completes)
// have rings of their own, four stages each, filled by two loader warps, so a
// stage is held only for as long as its operand is needed; items alternate
// between two softmax warp groups (warps 2-5: group 0, warps 6-9: group 1),
// each with one TMEM S buffer (P written over it) and two O buffers, and a
// group writes an item's output only after the softmax of its next item, so
// the PV MMA's latency is hidden.  One KV tile per item: plain softmax.  A
// warp whose 32 rows all lie at or past the sequence length (rows 96-127 for
// L = 90) does no softmax or output work: the rows of P it leaves stale only
// reach rows of O that are never stored.
constexpr int kItemThreads = 384;   // warps: Q/K loader, S issuer, 8 softmax, PV issuer, V loader
constexpr int kItemStages = 4;      // stages of each ring

struct ItemSmem {
  static constexpr int kQkStage = 2 * kQBytes;               // Q, K: 32 KB
  static constexpr int kV = kItemStages * kQkStage;           // V ring: kItemStages x 16 KB
  static constexpr int kOut = kV + kItemStages * kQBytes;     // per group: the gated output tile, 128 x 64 16-bit
  static constexpr int kOutBytes = kTile * kDimHead * 2;
  static constexpr int kBar = kOut + 2 * kOutBytes;
  static constexpr int kBytes = 1024 + kBar + 512;
};

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}
__device__ __forceinline__ void bulk_group_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_group_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_group_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Output row of query position `pos` of sequence `seq` (32-bit: rows < 2^31).
__device__ __forceinline__ int attn_row(const AttnArgs& args, int seq, int pos) {
  if (args.pos_dim == 1) return seq * args.d1 + pos;
  const int c_a = seq % args.d1;
  const int c_b = seq / args.d1;
  return (c_b * args.d2 + pos) * args.d1 + c_a;
}

template <typename T, int NCOLS>
__global__ void __launch_bounds__(kItemThreads, 1)
    attention_items_kernel(const __grid_constant__ CUtensorMap map, const __grid_constant__ CUtensorMap map_out,
                           const AttnArgs args) {
  static_assert(NCOLS % 32 == 0 && NCOLS <= kTile, "score columns per row");
  using L = ItemSmem;
  // TMEM columns: S/P of group g at [g * NCOLS, +NCOLS); O buffer b of group g
  // at [2 * NCOLS + 64 (2 g + b), +64).
  constexpr uint32_t kColO = 2 * NCOLS;
  static_assert(2 * NCOLS + 4 * kDimHead <= 512, "TMEM columns");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBar);
  uint64_t* qk_full = bars;                          // [stage]
  uint64_t* qk_free = bars + kItemStages;            // [stage]
  uint64_t* v_full = bars + 2 * kItemStages;         // [stage]
  uint64_t* v_free = bars + 3 * kItemStages;         // [stage]
  uint64_t* s_full = bars + 4 * kItemStages;         // [group]
  uint64_t* p_full = s_full + 2;                     // [group]
  uint64_t* o_full = p_full + 2;                     // [group][buffer]
  uint64_t* o_free = o_full + 4;                     // [group][buffer]
  uint64_t* drain = o_free + 4;                      // [issuer]
  uint64_t* out_free = drain + 2;                    // [group]: the output tile may be rewritten
  uint64_t* out_ready = out_free + 2;                // [group]: all rows of the output tile written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(out_ready + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = warp_id();
  const int lane = lane_id();
  const int length = args.length;
  const int nc = round16(length);
  const int total = args.sequences * kHeads;   // host checks < 2^31
  const int n_local = static_cast<int>(blockIdx.x) < total ? (total - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1 : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kItemStages; ++i) {
      mbar_init(&qk_full[i], 1);
      mbar_init(&qk_free[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_free[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 4);
    }
    mbar_init(drain, 1);
    mbar_init(drain + 1, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&out_free[i], 1);
      mbar_init(&out_ready[i], 4);
    }
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
  // Item k of this CTA: global item blockIdx.x + k * gridDim.x; head fastest.
  auto item_of = [&](int k) { return static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x); };

  if (warp == 0 || warp == 11) {
    // Loaders: warp 0 brings Q and K of each item into the Q/K ring, warp 11
    // brings V into the V ring; each waits only for its own ring's stage.
    if (lane == 0) {
      const bool qk = warp == 0;
      tma_prefetch(&map);
      if (qk) tma_prefetch(&map_out);
      for (int k = 0; k < n_local; ++k) {
        const int st = k % kItemStages;
        const uint32_t par = static_cast<uint32_t>(k / kItemStages) & 1u;
        if (!mbar_wait(qk ? &qk_free[st] : &v_free[st], par ^ 1u, abort_flag, args.err, kErrWaitTma)) break;
        const int item = item_of(k);
        const int head = item % kHeads;
        const int seq = item / kHeads;
        int c_a, c_b;
        if (args.pos_dim == 1) {
          c_a = seq % args.d2;
          c_b = seq / args.d2;
        } else {
          c_a = seq % args.d1;
          c_b = seq / args.d1;
        }
        uint64_t* bar = qk ? &qk_full[st] : &v_full[st];
        uint8_t* dst = qk ? smem + st * L::kQkStage : smem + L::kV + st * kQBytes;
        mbar_arrive_expect_tx(bar, qk ? 2 * kQBytes : kQBytes);
        for (int part = qk ? 0 : 2; part < (qk ? 2 : 3); ++part) {
          const int col = part * kDimInner + head * kDimHead;
          uint8_t* d = dst + (qk ? part * kQBytes : 0);
          if (args.pos_dim == 1)
            tma_load_4d(d, &map, bar, col, 0, c_a, c_b);
          else
            tma_load_4d(d, &map, bar, col, c_a, 0, c_b);
        }
      }
    }
  } else if (warp == 1) {
    // S issuer: S(k) = Q K^T as soon as item k's Q, K are in and group g's S
    // buffer is free (PV(k-2) has read the P that S(k) overwrites).  Item k:
    // group g = k & 1, group index i = k >> 1, O buffer b = i & 1.
    const uint32_t bf = ElemTraits<T>::kBf16;
    const uint32_t idesc_s = idesc_f16(kTile, static_cast<uint32_t>(nc), bf, 0, 0);
    const uint64_t base_desc_k = sw128_desc(smem_u32(smem), 16, 1024);
    bool ok = true;
    for (int k = 0; ok && k < n_local; ++k) {
      const int g = k & 1;
      const int i = k >> 1;
      const int st = k % kItemStages;
      if (!mbar_wait_warp(&qk_full[st], static_cast<uint32_t>(k / kItemStages) & 1u, abort_flag, args.err,
                          kErrWaitMma)) {
        ok = false;
        break;
      }
      if (i >= 1 && !mbar_wait_warp(&o_full[2 * g + ((i - 1) & 1)], static_cast<uint32_t>((i - 1) >> 1) & 1u,
                                    abort_flag, args.err, kErrWaitMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (elect_one()) {
        const uint64_t qd = base_desc_k + static_cast<uint64_t>((st * L::kQkStage) >> 4);
        const uint64_t kd = qd + static_cast<uint64_t>(kQBytes >> 4);
#pragma unroll
        for (int kk = 0; kk < kDimHead / 16; ++kk)
          umma_f16(tmem_base + g * NCOLS, qd + 2 * kk, kd + 2 * kk, idesc_s, kk != 0 ? 1u : 0u);
        umma_commit(&s_full[g]);
        umma_commit(&qk_free[st]);   // Q and K of this stage are read
      }
      __syncwarp();
    }
    if (elect_one()) {
      umma_commit(drain);
      wait_drain(drain, 0, args.err);
    }
    __syncwarp();
  } else if (warp == 10) {
    // PV issuer: O(k) = P(k) V as soon as item k's P is in TMEM, its V is in
    // and its O buffer was read (item k - 4); its commit frees the V stage.
    const uint32_t bf = ElemTraits<T>::kBf16;
    const uint32_t idesc_o = idesc_f16(kTile, kDimHead, bf, 0, 1);
    const uint64_t base_desc_v = sw128_desc(smem_u32(smem), 8192, 1024);
    for (int k = 0; k < n_local; ++k) {
      const int g = k & 1;
      const int i = k >> 1;
      const int ob = 2 * g + (i & 1);
      const int st = k % kItemStages;
      if (!mbar_wait_warp(&p_full[g], static_cast<uint32_t>(i) & 1u, abort_flag, args.err, kErrWaitMma)) break;
      if (i >= 2 && !mbar_wait_warp(&o_free[ob], static_cast<uint32_t>((i >> 1) - 1) & 1u, abort_flag, args.err,
                                    kErrWaitMma))
        break;
      if (!mbar_wait_warp(&v_full[st], static_cast<uint32_t>(k / kItemStages) & 1u, abort_flag, args.err,
                          kErrWaitMma))
        break;
      tc_fence_after();
      if (elect_one()) {
        const uint64_t vd = base_desc_v + static_cast<uint64_t>((L::kV + st * kQBytes) >> 4);
        const uint32_t p_col = tmem_base + g * NCOLS;
#pragma unroll
        for (int kk = 0; kk < NCOLS / 16; ++kk)
          if (kk * 16 < nc)
            umma_f16_ts(tmem_base + kColO + ob * kDimHead, p_col + kk * 8, vd + (kk * 2048 >> 4), idesc_o,
                        kk != 0 ? 1u : 0u);
        umma_commit(&o_full[ob]);
        umma_commit(&v_free[st]);
      }
      __syncwarp();
    }
    if (elect_one()) {
      umma_commit(drain + 1);
      wait_drain(drain + 1, 0, args.err);
    }
    __syncwarp();
  } else {
    const int g = (warp - 2) >> 2;
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const bool active = quarter * 32 < length;   // warp-uniform
    const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t s_addr = tmem_base + g * NCOLS + lane_off;
    // Output of the previous item of this group, written after the next
    // softmax: each warp puts its gated rows into the group's shared-memory
    // tile (128-byte swizzle) and one thread stores the tile with TMA (rows
    // past the sequence length fall outside the tensor map and are not
    // written).  out_free / out_ready hand the tile between the four warps
    // and that thread (quarter 0, lane 0), with bounded waits.
    int pend_k = -1;
    float pend_gate = 0.f, pend_sum = 1.f;
    int outputs = 0;   // tiles this group has stored
    uint8_t* out_tile = smem + L::kOut + g * L::kOutBytes;
    const bool issuer = quarter == 0 && lane == 0;
    auto write_output = [&]() -> bool {
      const int i = pend_k >> 1;
      const int ob = 2 * g + (i & 1);
      if (!mbar_wait_warp(&o_full[ob], static_cast<uint32_t>(i >> 1) & 1u, abort_flag, args.err, kErrWaitSoftmax))
        return false;
      tc_fence_after();
      uint32_t r0[32], r1[32];
      if (active) {
        const uint32_t o_addr = tmem_base + kColO + ob * kDimHead + lane_off;
        tmem_ld32(o_addr, r0);
        tmem_ld32(o_addr + 32, r1);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_free[ob]);
      // The tile is free once the previous store from it has read it.
      if (outputs > 0) {
        if (issuer) {
          bulk_group_wait_read_all();
          mbar_arrive(&out_free[g]);
        }
        if (!mbar_wait_warp(&out_free[g], static_cast<uint32_t>(outputs - 1) & 1u, abort_flag, args.err,
                            kErrWaitSoftmax))
          return false;
      }
      if (active && row < length) {
        const float scale = pend_gate / pend_sum;
        uint8_t* line = out_tile + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
        for (int gq = 0; gq < 8; ++gq) {
          const uint32_t* r = gq < 4 ? &r0[gq * 8] : &r1[(gq - 4) * 8];
          uint4 w;
          w.x = ElemTraits<T>::pack2(__uint_as_float(r[0]) * scale, __uint_as_float(r[1]) * scale);
          w.y = ElemTraits<T>::pack2(__uint_as_float(r[2]) * scale, __uint_as_float(r[3]) * scale);
          w.z = ElemTraits<T>::pack2(__uint_as_float(r[4]) * scale, __uint_as_float(r[5]) * scale);
          w.w = ElemTraits<T>::pack2(__uint_as_float(r[6]) * scale, __uint_as_float(r[7]) * scale);
          *reinterpret_cast<uint4*>(line + ((gq ^ (row & 7)) << 4)) = w;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&out_ready[g]);
      if (issuer) {
        if (!mbar_wait(&out_ready[g], static_cast<uint32_t>(outputs) & 1u, abort_flag, args.err, kErrWaitSoftmax))
          return false;
        const int item = item_of(pend_k);
        const int head = item % kHeads;
        const int seq = item / kHeads;
        if (args.pos_dim == 1)
          tma_store_4d(&map_out, out_tile, head * kDimHead, 0, seq % args.d2, seq / args.d2);
        else
          tma_store_4d(&map_out, out_tile, head * kDimHead, seq % args.d1, 0, seq / args.d1);
        bulk_group_commit();
      }
      ++outputs;
      return true;
    };
    bool ok = true;
    for (int k = g; ok && k < n_local; k += 2) {
      const int i = k >> 1;
      const int item = item_of(k);
      const int head = item % kHeads;
      const int out_row = (active && row < length) ? attn_row(args, item / kHeads, row) : 0;
      const float gate = (active && row < length) ? __ldg(args.gates + static_cast<long long>(out_row) * kHeads + head) : 0.f;
      if (!mbar_wait_warp(&s_full[g], static_cast<uint32_t>(i) & 1u, abort_flag, args.err, kErrWaitSoftmax)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sum = 1.0f;
      if (active) {
        // One pass over S in TMEM, 64 columns at a time.  Each chunk is
        // exponentiated against a reference maximum that only has to keep
        // exp2 below 2^8: it is raised -- and the packed P of earlier chunks
        // and the running sums rescaled -- only when a chunk exceeds it by
        // more than 2^8.  Columns >= length (stale, or never written by the
        // N = nc MMA) are masked.  P (two 16-bit values per column) goes over
        // the first NCOLS/2 columns of S once all of S is in registers.
        float m_ref = -INFINITY;
        float2 sums[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                          make_float2(0.f, 0.f)};
        uint32_t pk[NCOLS / 2];
#pragma unroll
        for (int c0 = 0; c0 < NCOLS; c0 += 64) {
          const int width = NCOLS - c0 < 64 ? NCOLS - c0 : 64;
          uint32_t ra[32], rb[32];
          tmem_ld32(s_addr + c0, ra);
          if (width == 64) tmem_ld32(s_addr + c0 + 32, rb);
          tmem_wait_ld();
          reg_fence(ra);
          if (width == 64) reg_fence(rb);
          float v[64];
#pragma unroll
          for (int q = 0; q < 64; ++q) {
            if (q < width) {
              const float x = __uint_as_float(q < 32 ? ra[q] : rb[q - 32]);
              v[q] = c0 + q < length ? x : -INFINITY;
            }
          }
          float mxs[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) mxs[e] = v[e];
#pragma unroll
          for (int q = 8; q < 64; q += 16) {
            if (q + 16 <= width) {
#pragma unroll
              for (int e = 0; e < 8; ++e) mxs[e] = fmax3(mxs[e], v[q + e], v[q + 8 + e]);
            }
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) mxs[e] = fmaxf(mxs[e], v[width - 8 + e]);   // last 8 columns of the chunk
          const float mx =
              fmax3(fmax3(mxs[0], mxs[1], mxs[2]), fmax3(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
          if ((mx - m_ref) * kScaleLog2 > kRescaleLog2) {
            const float f = ex2_approx((m_ref - mx) * kScaleLog2);   // 0 when m_ref = -inf
            m_ref = mx;
            const float2 f2 = make_float2(f, f);
#pragma unroll
            for (int e = 0; e < 4; ++e) sums[e] = __fmul2_rn(sums[e], f2);
            if (c0 > 0) {
              const uint32_t fp = ElemTraits<T>::pack2(f, f);
#pragma unroll
              for (int q = 0; q < c0 / 2; ++q) pk[q] = ElemTraits<T>::mul2(pk[q], fp);
            }
          }
          const float mscaled = m_ref * kScaleLog2;
          const float2 c2 = make_float2(kScaleLog2, kScaleLog2);
          const float2 nm2 = make_float2(-mscaled, -mscaled);
#pragma unroll
          for (int q = 0; q < 64; q += 2) {
            if (q < width) {
              const float2 x2 = __ffma2_rn(make_float2(v[q], v[q + 1]), c2, nm2);
              float2 p2;
              if (((q >> 1) & 7) < kItemPolyPairs) {
                p2 = exp2_poly2(x2);
              } else {
                p2.x = ex2_approx(x2.x);
                p2.y = ex2_approx(x2.y);
              }
              sums[(q >> 1) & 3] = __fadd2_rn(sums[(q >> 1) & 3], p2);
              pk[(c0 + q) / 2] = ElemTraits<T>::pack2(p2.x, p2.y);
            }
          }
        }
#pragma unroll
        for (int c = 0; c < NCOLS / 64; ++c) {
          uint32_t w[32];
#pragma unroll
          for (int q = 0; q < 32; ++q) w[q] = pk[32 * c + q];
          tmem_st32(s_addr + 32 * c, w);
        }
        if (NCOLS % 64 == 32) {
          uint32_t w[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) w[q] = pk[NCOLS / 2 - 16 + q];
          tmem_st16(s_addr + NCOLS / 2 - 16, w);
        }
        const float2 s01 = __fadd2_rn(__fadd2_rn(sums[0], sums[1]), __fadd2_rn(sums[2], sums[3]));
        sum = s01.x + s01.y;
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[g]);
      if (pend_k >= 0 && !write_output()) {
        ok = false;
        break;
      }
      pend_k = k;
      pend_gate = gate;
      pend_sum = sum;
    }
    if (ok && pend_k >= 0) write_output();
    if (issuer) bulk_group_wait_all();   // every tile store has completed before the CTA exits
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <typename T, int NCOLS>
cudaError_t launch_items_cols(const CUtensorMap& map, const AttnArgs& args, int sm_count, cudaStream_t stream) {
  static std::atomic<unsigned long long> configured{0};
  const cudaError_t e = opt_in_smem(attention_items_kernel<T, NCOLS>, ItemSmem::kBytes, configured);
  if (e != cudaSuccess) return e;
  const long long items = static_cast<long long>(args.sequences) * kHeads;
  if (items <= 0) return cudaSuccess;
  // Gated output [rows][512] viewed like the qkv map: (512, d1, d2, d3), one
  // 64-column head by up to 128 positions per store.
  const long long rows_all = static_cast<long long>(args.sequences) * args.length;
  const long long d3 = rows_all / (static_cast<long long>(args.d1) * args.d2);
  const uint64_t dims[4] = {static_cast<uint64_t>(kDimInner), static_cast<uint64_t>(args.d1),
                            static_cast<uint64_t>(args.d2), static_cast<uint64_t>(d3)};
  const uint64_t rb = kDimInner * 2ull;
  const uint64_t strides[3] = {rb, rb * args.d1, rb * args.d1 * args.d2};
  const uint32_t box[4] = {64u, args.pos_dim == 1 ? 128u : 1u, args.pos_dim == 2 ? 128u : 1u, 1u};
  CUtensorMap map_out;
  if (!make_tmap_4d(&map_out, args.out, 2, dims, strides, box, ElemTraits<T>::kBf16 != 0)) return cudaErrorInvalidValue;
  // The kernel indexes items and output rows in 32 bits.
  const long long rows = static_cast<long long>(args.sequences) * args.length;
  if (items > 0x7FFFFFFFLL || rows > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const int grid = items < sm_count ? static_cast<int>(items) : sm_count;
  attention_items_kernel<T, NCOLS><<<grid, kItemThreads, ItemSmem::kBytes, stream>>>(map, map_out, args);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_items(const CUtensorMap& map, const AttnArgs& args, int sm_count, cudaStream_t stream) {
  return args.length <= 96 ? launch_items_cols<T, 96>(map, args, sm_count, stream)
                           : launch_items_cols<T, 128>(map, args, sm_count, stream);
}

}  // namespace

cudaError_t launch_attention(bool bf16, const CUtensorMap& map_qkv, const AttnArgs& args, int sm_count,
                             cudaStream_t stream) {
  // Single-tile sequences (band axis, L <= 128): persistent two-slot item
  // kernel.  Longer sequences: two query tiles per CTA.
  const bool single = args.length <= kTile;
  if (bf16)
    return single ? launch_items<__nv_bfloat16>(map_qkv, args, sm_count, stream)
                  : launch_pair<__nv_bfloat16>(map_qkv, args, sm_count, stream);
  return single ? launch_items<__half>(map_qkv, args, sm_count, stream)
                : launch_pair<__half>(map_qkv, args, sm_count, stream);
}

}  // namespace vab
