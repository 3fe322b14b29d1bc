// Internal declarations shared by the sm_100a kernels and the runtime.
#pragma once

#include <atomic>
#include <vector>
#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace vab {

// Model constants of the bundled BS-RoFormer (native/vocalarc_separation.c:33-46).
constexpr int kDim = 256;
constexpr int kDepth = 16;
constexpr int kBands = 90;
constexpr int kHeads = 8;
constexpr int kDimHead = 64;
constexpr int kDimInner = 512;
constexpr int kQkvDim = 1536;
constexpr int kFfDim = 1024;
constexpr int kFreqBins = 1025;
constexpr int kChannels = 2;
constexpr int kNfft = 2048;
constexpr int kHop = 512;
constexpr int kModelFrames = 1722;
constexpr int kBandSplitDim = 4100;  // sum of 4 * band width

// A kernel's opt-in to more than 48 KB of dynamic shared memory
// (cudaFuncSetAttribute) holds for the current device only, so it is made
// once per device: bit d of `done` records device d.  A process that drives
// several GPUs (one provider each) needs it on every one of them.
template <typename K>
inline cudaError_t opt_in_smem(K* kernel, int bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = dev >= 0 && dev < 64 ? (1ull << dev) : 0ull;
  if (bit != 0 && (done.load(std::memory_order_relaxed) & bit) != 0) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_relaxed);
  return e;
}

// ------------------------------------------------------------------ GEMM
enum EpilogueKind : int {
  kEpiStore = 0,      // out_16[r][n] = acc * inv[r] (+ bias[n])            (staged TMA store)
  kEpiGelu = 1,       // out_16[r][n] = gelu(acc * inv[r] + bias[n])         (staged TMA store)
  kEpiQkvRope = 2,    // out_16 = RoPE(acc * inv[r]) on q and k; gate tile -> sigmoid gates
  kEpiResidual = 3,   // resid_f32 += acc (+ bias); x16 = resid; row_inv_out = sqrt(256)/|resid|
  kEpiTanhBand = 4,   // grouped mask layer 1: out_16[r][n0+c] = tanh(acc * inv[r] + bias[b_row + c])
  kEpiGluMask = 5,    // grouped mask layer 2: GLU pairs scattered into the complex mask
  kEpiStoreF32 = 6,   // out_f32[r][n] = acc (tests)
  kEpiGeglu = 7,      // columns interleave (value i, gate i): out_16[r][n/2] = value * gelu(gate), both
                      // acc * inv[r] + bias (staged TMA store)
};

// Tensor maps of one GEMM launch: A and B operands; c = the staged output
// (16-bit [rows][N], box 64x32, 128B swizzle; or the fp32 residual, box 32x32,
// 128B swizzle); d = the 16-bit copy of the residual (box 32x32, 64B swizzle).
struct GemmMaps {
  CUtensorMap a, b, c, d;
};

struct GemmArgs {
  int m_rows;           // uniform: valid rows of A
  int n_tiles;          // uniform: N / 256 (full-width tiles)
  int gate_tile;        // uniform: 1 = one extra 16-column tile after the n_tiles (QKV gate logits)
  int k_blocks;         // K / 64
  int num_tiles;        // total tiles
  const int4* tiles;    // grouped: per-chunk tile table {a_row, b_row, n0, meta}
  int tiles_per_chunk;  // grouped: entries of the table
  int chunk_rows;       // grouped: A-row offset between chunk replicas
  int b_box16;          // 1: B loaded as n_size/16 boxes of 16 rows
  void* out;            // direct epilogues
  long long ldo;
  const float* bias;
  const float* row_inv;  // per-row RMSNorm factor applied to the accumulator (null = 1)
  float* row_inv_out;    // kEpiResidual: per-row factor of the updated residual
  // RoPE (cos, sin) in slot-major order: rope[q * rope_stride + pos] holds
  // pairs 2q and 2q + 1 of position pos, so the 32 rows of a warp (consecutive
  // positions on the time axis) read 512 contiguous bytes per slot.
  const float4* rope;
  int rope_stride;
  int pos_div;
  int pos_mod;
  int rope_cols;
  const float* gate_b;  // QKV gate tile: [8]
  float* gates_out;     // QKV gate tile: [rows][8]
  int frames;           // mask: frames per chunk (T)
  int mask_ref_layout;  // mask: 1 = reference [1025][2][T][2], 0 = frame-major [C][T][1025][2][2]
  int* err;
  // kEpiResidual over N > 256: each column tile adds its share of sum x^2 to
  // row_sumsq_out[r] (zeroed beforehand; two tiles per row add in either order
  // to the same float) instead of writing row_inv_out.
  float* row_sumsq_out;
  // kEpiGluMask for a model other than the bundled one: band count and the
  // per-band first bin / 4 * width tables in global memory (0 / null = the
  // bundled 90-band tables).
  int bands;
  const int* band_first;
  const int* band_dim;
  // launch_ffn: the FFN input bias b1 (bias = the output bias b2).
  const float* bias1;
};

// Grouped-tile metadata packing: m_valid (8 bits) | n_size (9 bits) << 8 | band << 17.
inline int4 make_tile(int a_row, int b_row, int n0, int m_valid, int n_size, int band) {
  return make_int4(a_row, b_row, n0, m_valid | (n_size << 8) | (band << 17));
}

// 2-D map over a row-major [outer][inner] matrix of 16-bit (bf16 or f16) or
// fp32 (elem_bytes 4) elements; swizzle_bytes 0, 64 or 128.
bool make_tmap_2d(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer, int swizzle_bytes,
                  bool bf16);
bool make_tmap_4d(CUtensorMap* map, const void* base, int elem_bytes, const uint64_t dims[4],
                  const uint64_t strides_bytes[3], const uint32_t box[4], bool bf16);

// Launches the persistent tcgen05 GEMM  C = A[M][K] * B[N][K]^T  with the given
// epilogue.  A and B are 16-bit (f16 or bf16 per `bf16`).
cudaError_t launch_gemm(int epilogue, bool bf16, const GemmMaps& maps, const GemmArgs& args, int sm_count,
                        cudaStream_t stream);

// The whole feed-forward sub-block of a width-256 row in one kernel:
//   x += GELU(inv * x16 W1^T + b1) W2^T + b2, then x16 and inv of the new x.
// The hidden activations stay on chip.  x16: 16-bit rows, box 64x128, 128B
// swizzle; w1: W1 [F][256], box 64x128; w2: W2 [256][F], box 64x256; res: fp32
// x, box 32x32, 128B swizzle; out16: x16 again, box 32x32, 64B swizzle.
struct FfnMaps {
  CUtensorMap x16, w1, w2, res, out16;
};
// args: m_rows, num_tiles (= ceil(m_rows / 128)), row_inv (read), row_inv_out
// (written), bias1 = b1, bias = b2, out = the fp32 x (for an L2 prefetch), err.
// hidden = F (a multiple of 128).
cudaError_t launch_ffn(bool bf16, const FfnMaps& maps, const GemmArgs& args, int hidden, int sm_count,
                       cudaStream_t stream);

// ------------------------------------------------------------------ attention
struct AttnArgs {
  int length;       // L, positions per sequence
  int sequences;    // S
  int q_tiles;      // ceil(L / 128)
  int pos_dim;      // 1: positions along tensor-map dim 1, 2: along dim 2
  int d1, d2;       // tensor-map extents of dims 1 and 2 (rows = (d3 * d2 + i2) * d1 + i1)
  const float* gates;  // [rows][8] sigmoid gates
  void* out;           // [rows][512] gated attention output (16-bit)
  int* err;
};
cudaError_t launch_attention(bool bf16, const CUtensorMap& map_qkv, const AttnArgs& args, int sm_count,
                             cudaStream_t stream);

// ------------------------------------------------------------------ elementwise / spectral
struct SegmentMap {
  // Where sample i of segment c comes from (see segment_sample in spectral.cu).
  int mode;          // 0 = whole clip (segment c = clip c), 1 = demix chunks of one clip
  int clip_length;   // samples per channel of the input clip(s)
  int seg_length;    // samples per segment (whole: clip_length, demix: chunk size)
  int border;        // demix: reflect border (0 when the clip is not padded)
  int padded;        // demix: padded working length
  int step;          // demix: chunk step
  long long clip_stride;  // whole mode: floats between clips
  int first_chunk;   // demix: global index of segment 0 of this pass
};

inline SegmentMap whole_clip_map(int length) {
  return SegmentMap{0, length, length, 0, length, 0, 2ll * length, 0};
}
inline SegmentMap demix_map(int length, int chunk, int border, int padded, int step, int first_chunk) {
  return SegmentMap{1, length, chunk, border, padded, step, 0, first_chunk};
}

cudaError_t launch_stft(const float* audio, SegmentMap map, int segments, int frames,
                        const float* window, const float2* twiddle, float* spec, cudaStream_t stream,
                        int hop = kHop);
// Band split into `dim` (256 or 512) columns over `bands` bands; x rows are
// (segment * bands + band) * frames + frame.
cudaError_t launch_band_split(const float* spec, int segments, int frames, const float* band_wt,
                              const long long* band_wt_offset, const float* band_gamma,
                              const int* band_gamma_offset, const float* band_bias, float* x,
                              cudaStream_t stream, int dim = kDim, int bands = kBands);
// Row statistics of a [rows][dim] fp32 residual (dim 256 or 512): x16 and
// inv = sqrt(dim) / sqrt(sum x^2 + 1e-12).
cudaError_t launch_row_stats_dim(const float* x, long long rows, int dim, void* x16, float* inv, bool bf16,
                                 cudaStream_t stream);
// inv[r] = scale / sqrt(sumsq[r] + 1e-12), then sumsq[r] = 0.
cudaError_t launch_norm_finalize(float* sumsq, float* inv, long long rows, float scale, cudaStream_t stream);
// Row statistics of the fp32 residual: x16 = 16-bit copy of x and
// inv = sqrt(256) / sqrt(sum x^2 + 1e-12) per row.  With remap_s0 > 0 the rows
// of a physical [remap_s0][remap_l0] token grid are written as [l0][s0].
cudaError_t launch_row_stats(const float* x, long long rows, void* x16, float* inv, bool bf16, int remap_s0,
                             int remap_l0, cudaStream_t stream);
cudaError_t launch_istft_frames(const float* spec, const float* mask, int segments, int frames,
                                const float* window, const float2* twiddle, float* frames_out,
                                cudaStream_t stream);
cudaError_t launch_overlap_add(const float* frames_buf, int segments, int frames, int seg_length,
                               const float* window, float* seg_out, cudaStream_t stream, int hop = kHop);
cudaError_t launch_demix(const float* seg_out, SegmentMap map, int chunks, int model_batch,
                         float* vocals, cudaStream_t stream);
// One contiguous chunk range of a track sharded across GPUs: padded samples
// [p0, p1), accumulators initialised from `init` ([3][init_len]: channel 0,
// channel 1, weight; padded sample init_p0 first) where present.  Writes the
// partial sums to seam_out ([3][p1 - p0]) when set, else the divided, cropped
// samples to vocals ([2][clip_length]).
struct DemixRange {
  int c0, c1;
  int p0, p1;
  const float* init;
  int init_p0, init_len;
  float* seam_out;
  float* vocals;
};
cudaError_t launch_demix_range(const float* seg_out, SegmentMap map, int chunks, int model_batch,
                               const DemixRange& range, cudaStream_t stream);
// Bigshift + TTA variants of a mix ([variants][shifts][2][n]) and the
// reference-order combination of their estimates into vocals [2][n].
cudaError_t launch_tta_inputs(const float* mix, int n, int shifts, int variants, float* out, cudaStream_t stream);
cudaError_t launch_tta_combine(const float* est, int n, int shifts, int tta, float* vocals, cudaStream_t stream);
cudaError_t launch_transpose_tokens(const float* src, float* dst, int s0, int l0, cudaStream_t stream);
// ---- one axial block (block.cu), shared by the provider and the configurable stack
// Token grid (d1, d2, d3): row = (i3 * d2 + i2) * d1 + i1.  Attention runs
// along dim `pos_dim` over `sequences` sequences of `length` tokens; the RoPE
// position of row r is (r / pos_div) % pos_mod.
struct AxisPlan {
  int pos_dim, d1, d2, d3, sequences, length, pos_div, pos_mod;
};
// B-operand maps and vectors of one block's weights (norm gammas folded in).
struct AxialWeights {
  const CUtensorMap* m_qkv;
  const CUtensorMap* m_out;
  const CUtensorMap* m_ff1;
  const CUtensorMap* m_ff2;
  const void* ff1_w;  // W1 itself (the fused FFN maps it in 128-row boxes)
  const float* gate_b;
  const float* ff1_b;
  const float* ff2_b;
};
// The residual stream (fp32 x, its 16-bit copy, the per-row RMSNorm factor)
// and the block's operand buffers; `wide` holds q|k|v [tokens][1536], later
// the FFN hidden.  sumsq: width > 256 only (zero between uses).
struct AxialBuffers {
  float* x;
  void* x16;
  float* row_inv;
  float* sumsq;
  void* wide;
  void* attn;
  float* gates;
  const float4* rope;   // slot-major RoPE table (rope_table), rope_stride positions
  int* err;
  int rope_stride;
};
// The RoPE (cos, sin) table for positions [0, n) in the slot-major layout the
// QKV epilogue reads (GemmArgs::rope): n * 16 float4.
std::vector<float4> rope_table(int n);

struct AxialShape {
  int dim;        // 256 or 512
  int ff_inner;   // FFN hidden width
  int geglu;      // 1: the FFN input GEMM emits interleaved (value, gate) rows
};
// The owner's launch bookkeeping (error check, launch count, trace mark).
using LaunchHook = bool (*)(void* owner, cudaError_t e, const char* what);
// Needs x16 / row_inv of the current x and the RoPE table for ax.length
// positions; leaves them describing the updated x.
bool run_axial_block(const AxialBuffers& b, const AxialWeights& w, const AxialShape& sh, long long tokens,
                     const AxisPlan& ax, bool bf16, int sm_count, cudaStream_t stream, LaunchHook hook, void* owner);

// One CTA waiting, with the kernels' wait loop and the given limit, on an
// mbarrier that never completes; records kErrWaitTma in *err and returns.
cudaError_t launch_wait_check(int* err, unsigned long long limit_ns, cudaStream_t stream);
cudaError_t upload_band_tables(const int* first, const int* dims);

}  // namespace vab
