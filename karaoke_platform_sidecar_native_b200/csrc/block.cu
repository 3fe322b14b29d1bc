// One pre-norm axial transformer block on the device: the single orchestration
// shared by the bundled provider (runtime.cu) and the configurable stack
// (stack.cu).  transformer_forward, native/vocalarc_separation.c:836-873:
//   x += Out(Gate(Attn(RoPE(QKV(RMSNorm x)))));  x += FF2(act(FF1(RMSNorm x)))
// as four or five launches: the QKV GEMM (RoPE, row scale and the head-gate tile in
// its epilogue), tcgen05 attention with the gate in its output stage, the
// out-projection GEMM with the fp32 residual and the new row statistics, and
// the FFN: for width 256 with GELU one fused kernel that keeps the hidden on
// chip, otherwise the FFN input GEMM (bias + GELU, or GEGLU) and the FFN output
// GEMM with the residual and row statistics.  RMSNorm gammas are folded into
// the weights.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "vab_internal.h"

namespace vab {

namespace {

bool rows_map(CUtensorMap* map, const void* base, long long rows, int k, bool bf16) {
  return make_tmap_2d(map, base, 2, static_cast<uint64_t>(k), static_cast<uint64_t>(rows),
                      static_cast<uint64_t>(k) * 2, 64, 128, 128, bf16);
}

bool out16_map(CUtensorMap* map, const void* base, long long rows, int n, bool bf16) {
  return make_tmap_2d(map, base, 2, static_cast<uint64_t>(n), static_cast<uint64_t>(rows),
                      static_cast<uint64_t>(n) * 2, 64, 32, 128, bf16);
}

GemmArgs block_args(const AxialBuffers& b, long long rows, int n, int k) {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.m_rows = static_cast<int>(rows);
  a.n_tiles = n / 256;
  a.k_blocks = k / 64;
  a.num_tiles = static_cast<int>((rows + 127) / 128) * a.n_tiles;
  a.err = b.err;
  a.pos_div = 1;
  a.pos_mod = 1;
  return a;
}

// VOCALARC_B200_FFN=split selects the two-launch FFN (FF1 writes the hidden to
// HBM, FF2 reads it back) where the fused kernel applies; both compute the same
// products in the same order per output element up to the hidden's rounding.
bool ffn_fused_enabled() {
  static const bool fused = [] {
    const char* v = getenv("VOCALARC_B200_FFN");
    return v == nullptr || strcmp(v, "split") != 0;
  }();
  return fused;
}

}  // namespace

// cos/sin exactly as apply_rotary builds them (vocalarc_separation.c:726-731,
// frequencies from fill_frequencies :1312-1314), float arithmetic and libm;
// slot q of position p holds pairs 2q and 2q + 1.
std::vector<float4> rope_table(int n) {
  std::vector<float4> table(static_cast<size_t>(n) * 16);
  float freq[32];
  for (int i = 0; i < 32; ++i) freq[i] = 1.0f / powf(10000.0f, static_cast<float>(2 * i) / kDimHead);
  for (int p = 0; p < n; ++p)
    for (int q = 0; q < 16; ++q) {
      const float a0 = static_cast<float>(p) * freq[2 * q];
      const float a1 = static_cast<float>(p) * freq[2 * q + 1];
      table[static_cast<size_t>(q) * n + p] = make_float4(cosf(a0), sinf(a0), cosf(a1), sinf(a1));
    }
  return table;
}

bool run_axial_block(const AxialBuffers& b, const AxialWeights& w, const AxialShape& sh, long long tokens,
                     const AxisPlan& ax, bool bf16, int sm_count, cudaStream_t stream, LaunchHook hook,
                     void* owner) {
  const int d = sh.dim;
  GemmMaps maps;
  // q|k|v = RoPE(inv * x16 (gamma o Wqkv)^T), gates = sigmoid(inv * x16 (gamma o Wg)^T + b)
  if (!rows_map(&maps.a, b.x16, tokens, d, bf16) || !out16_map(&maps.c, b.wide, tokens, kQkvDim, bf16)) return false;
  maps.b = *w.m_qkv;
  maps.d = maps.c;
  GemmArgs args = block_args(b, tokens, kQkvDim, d);
  args.gate_tile = 1;
  args.num_tiles = static_cast<int>((tokens + 127) / 128) * (args.n_tiles + 1);
  args.row_inv = b.row_inv;
  args.rope = b.rope;
  args.rope_stride = b.rope_stride;
  args.pos_div = ax.pos_div;
  args.pos_mod = ax.pos_mod;
  args.rope_cols = 2 * kDimInner;
  args.gate_b = w.gate_b;
  args.gates_out = b.gates;
  if (!hook(owner, launch_gemm(kEpiQkvRope, bf16, maps, args, sm_count, stream), "qkv gemm")) return false;

  // Attention over the token grid (d1, d2, d3) along pos_dim; no transposes.
  CUtensorMap q4;
  const uint64_t dims[4] = {static_cast<uint64_t>(kQkvDim), static_cast<uint64_t>(ax.d1),
                            static_cast<uint64_t>(ax.d2), static_cast<uint64_t>(ax.d3)};
  const uint64_t row_bytes = kQkvDim * 2ull;
  const uint64_t strides[3] = {row_bytes, row_bytes * ax.d1, row_bytes * ax.d1 * ax.d2};
  const uint32_t box[4] = {64u, ax.pos_dim == 1 ? 128u : 1u, ax.pos_dim == 2 ? 128u : 1u, 1u};
  if (!make_tmap_4d(&q4, b.wide, 2, dims, strides, box, bf16)) return false;
  AttnArgs at;
  at.length = ax.length;
  at.sequences = ax.sequences;
  at.q_tiles = (ax.length + 127) / 128;
  at.pos_dim = ax.pos_dim;
  at.d1 = ax.d1;
  at.d2 = ax.d2;
  at.gates = b.gates;
  at.out = b.attn;
  at.err = b.err;
  if (!hook(owner, launch_attention(bf16, q4, at, sm_count, stream),
            ax.length <= 128 ? "attention (L<=128)" : "attention (L>128)"))
    return false;

  // x += A W^T (+ bias), with x16 and the row factor of the new x.  Width 256
  // is one column tile, which writes the factor itself; wider rows gather
  // their sum of squares over the column tiles and finish it in one pass.
  auto residual = [&](const CUtensorMap& map_a, const CUtensorMap& map_b, int k, const float* bias,
                      const char* what) {
    GemmMaps rm;
    rm.a = map_a;
    rm.b = map_b;
    if (!make_tmap_2d(&rm.c, b.x, 4, d, static_cast<uint64_t>(tokens), d * 4ull, 32, 32, 128, false) ||
        !make_tmap_2d(&rm.d, b.x16, 2, d, static_cast<uint64_t>(tokens), d * 2ull, 32, 32, 64, bf16))
      return false;
    GemmArgs ra = block_args(b, tokens, d, k);
    ra.bias = bias;
    if (d == 256) {
      ra.row_inv_out = b.row_inv;
      return hook(owner, launch_gemm(kEpiResidual, bf16, rm, ra, sm_count, stream), what);
    }
    ra.row_sumsq_out = b.sumsq;
    return hook(owner, launch_gemm(kEpiResidual, bf16, rm, ra, sm_count, stream), what) &&
           hook(owner, launch_norm_finalize(b.sumsq, b.row_inv, tokens, sqrtf(static_cast<float>(d)), stream),
                "norm finalize");
  };

  CUtensorMap a_attn, a_x16, a_hidden;
  if (!rows_map(&a_attn, b.attn, tokens, kDimInner, bf16) ||
      !residual(a_attn, *w.m_out, kDimInner, nullptr, "out gemm"))
    return false;

  // x += GELU(inv * x16 (ff_gamma o W1)^T + b1) W2^T + b2 in one kernel, the
  // hidden on chip (width 256, GELU).
  if (d == 256 && !sh.geglu && sh.ff_inner % 128 == 0 && w.ff1_w != nullptr && ffn_fused_enabled()) {
    FfnMaps fm;
    if (!rows_map(&fm.x16, b.x16, tokens, d, bf16) ||
        !make_tmap_2d(&fm.w1, w.ff1_w, 2, d, static_cast<uint64_t>(sh.ff_inner), d * 2ull, 64, 128, 128, bf16) ||
        !make_tmap_2d(&fm.res, b.x, 4, d, static_cast<uint64_t>(tokens), d * 4ull, 32, 32, 128, false) ||
        !make_tmap_2d(&fm.out16, b.x16, 2, d, static_cast<uint64_t>(tokens), d * 2ull, 32, 32, 64, bf16))
      return false;
    fm.w2 = *w.m_ff2;
    GemmArgs fa = block_args(b, tokens, d, d);
    fa.num_tiles = static_cast<int>((tokens + 127) / 128);
    fa.row_inv = b.row_inv;
    fa.row_inv_out = b.row_inv;
    fa.bias1 = w.ff1_b;
    fa.bias = w.ff2_b;
    fa.out = b.x;
    return hook(owner, launch_ffn(bf16, fm, fa, sh.ff_inner, sm_count, stream), "ffn");
  }

  // hidden = GELU(inv * x16 (ff_gamma o W1)^T + b1), or GEGLU over interleaved (value, gate) rows.
  if (!rows_map(&a_x16, b.x16, tokens, d, bf16) || !out16_map(&maps.c, b.wide, tokens, sh.ff_inner, bf16))
    return false;
  maps.a = a_x16;
  maps.b = *w.m_ff1;
  maps.d = maps.c;
  args = block_args(b, tokens, sh.geglu ? 2 * sh.ff_inner : sh.ff_inner, d);
  args.row_inv = b.row_inv;
  args.bias = w.ff1_b;
  if (!hook(owner, launch_gemm(sh.geglu ? kEpiGeglu : kEpiGelu, bf16, maps, args, sm_count, stream), "ff1 gemm"))
    return false;

  // x += hidden W2^T + b2
  return rows_map(&a_hidden, b.wide, tokens, sh.ff_inner, bf16) &&
         residual(a_hidden, *w.m_ff2, sh.ff_inner, w.ff2_b, "ff2 gemm");
}

}  // namespace vab
