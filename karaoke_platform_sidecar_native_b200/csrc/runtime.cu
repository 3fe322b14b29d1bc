// Host runtime of the sm_100a provider: device context, weight conversion,
// workspace, forward orchestration and the C ABI (native_gpu.h plus the
// additive vocalarc_b200.h extension).
//
// Layout in HBM: the residual stream is one fp32 token matrix in band-major
// order, rows (segment * 90 + band) * T + frame, 256 columns.  Both axial
// blocks run on that same buffer: GEMMs are row-wise, and the attention
// kernel addresses a sequence (a band over time, or a frame over bands)
// through a 4-D TMA tensor map, so the reference's transpose kernels
// (native_gpu_cuda.cu:428-451) disappear.  16-bit copies feed the tensor
// cores (x, q/k/v, gated attention, FFN hidden); the mask head reads the
// band-major rows directly as its per-band A operand.  Every RMSNorm gamma is
// folded into the weights of the GEMM that consumes the norm, and the GEMM
// that updates x writes the per-row factor sqrt(256)/|x| next to x16.
#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "vab_internal.h"
#include "vocalarc_b200.h"

using namespace vab;

namespace {

const int kBandFreqs[kBands] = {
    2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,  2,
    4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,
    4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  4,  12, 12, 12, 12, 12, 12, 12, 12, 12, 12, 12, 12,
    12, 12, 12, 12, 24, 24, 24, 24, 24, 24, 24, 24, 48, 48, 48, 48, 128, 129};

int band_first(int band) {
  int f = 0;
  for (int b = 0; b < band; ++b) f += kBandFreqs[b];
  return f;
}
int round16(int x) { return (x + 15) & ~15; }

bool env_is_off(const char* name) {
  const char* v = getenv(name);
  return v != nullptr && (strcmp(v, "0") == 0 || strcmp(v, "false") == 0 || strcmp(v, "off") == 0);
}

// ------------------------------------------------------------------ weights
// Unpacks the reference's 32-lane packed layout (vocalarc_separation.c:428-457)
// into W[out][in].
void unpack_packed(const float* packed, int in, int out, std::vector<float>& w) {
  w.assign(static_cast<size_t>(in) * out, 0.f);
  const int full = (out / 32) * 32;
  for (int tile = 0; tile < full; tile += 32) {
    const float* src = packed + static_cast<size_t>(tile / 32) * in * 32;
    for (int i = 0; i < in; ++i)
      for (int lane = 0; lane < 32; ++lane) w[static_cast<size_t>(tile + lane) * in + i] = src[static_cast<size_t>(i) * 32 + lane];
  }
  if (full < out) {
    const int tail = out - full;
    const float* src = packed + static_cast<size_t>(out / 32) * in * 32;
    for (int i = 0; i < in; ++i)
      for (int lane = 0; lane < tail; ++lane) w[static_cast<size_t>(full + lane) * in + i] = src[static_cast<size_t>(i) * tail + lane];
  }
}

void to16(const std::vector<float>& w, bool bf16, std::vector<uint16_t>& out) {
  out.resize(w.size());
  for (size_t i = 0; i < w.size(); ++i) {
    if (bf16) {
      __nv_bfloat16 h = __float2bfloat16_rn(w[i]);
      memcpy(&out[i], &h, 2);
    } else {
      __half h = __float2half_rn(w[i]);
      memcpy(&out[i], &h, 2);
    }
  }
}

uint64_t fingerprint(const float* p, size_t n) {
  uint64_t h = 1469598103934665603ull ^ reinterpret_cast<uintptr_t>(p) ^ (n * 1099511628211ull);
  const size_t picks[8] = {0, 1, 2, 3, n / 2, n - 3, n - 2, n - 1};
  for (size_t i = 0; i < 8; ++i) {
    uint32_t bits;
    memcpy(&bits, p + (picks[i] < n ? picks[i] : 0), 4);
    h = (h ^ bits) * 1099511628211ull;
  }
  return h;
}

struct DeviceBuffer {
  void* ptr = nullptr;
  size_t bytes = 0;
};

// Device weights of one axial block.  qkv holds 1552 rows: the 1536 q|k|v
// rows and the 8 head-gate rows, both scaled column-wise by the attention
// RMSNorm gamma, then 8 zero rows; ff1 is scaled by the FF RMSNorm gamma.
constexpr int kQkvRows = kQkvDim + 16;
struct BlockW {
  void* qkv = nullptr;
  void* out = nullptr;
  void* ff1 = nullptr;
  void* ff2 = nullptr;
  float* gate_b = nullptr;
  float* ff1_b = nullptr;
  float* ff2_b = nullptr;
  CUtensorMap m_qkv, m_out, m_ff1, m_ff2;
};

struct CachedBlock {
  native_gpu_transformer_weights key;
  uint64_t print = 0;
  int bf16 = 0;
  void* mem = nullptr;
  BlockW w;
};

struct MaskW {
  void* w1 = nullptr;
  float* b1 = nullptr;
  void* w2 = nullptr;
  float* b2 = nullptr;
  int w2_off[kBands];
  int w2_rows[kBands];
  int w2_total = 0;
  CUtensorMap m_w1, m_w2;
};

struct BandW {
  float* wt = nullptr;          // per band [d_b][256]
  long long* wt_off = nullptr;  // [90]
  float* gamma = nullptr;       // [4100]
  int* gamma_off = nullptr;     // [91]
  float* bias = nullptr;        // [90][256]
};

// Bump allocator over one cudaMalloc.  With `host` set, weights are written
// to a host mirror of [base, base + cap) and reach the device in one copy
// later; with `dry` set, only pointers (and tensor maps) are laid out.
struct Arena {
  char* base = nullptr;
  size_t cap = 0, used = 0;
  uint8_t* host = nullptr;
  bool dry = false;
  bool maps = true;
  uint64_t layout = 1469598103934665603ull;   // hash of every (offset, size) taken
  void* take(size_t bytes) {
    const size_t off = (used + 1023) & ~size_t(1023);
    if (off + bytes > cap) return nullptr;
    used = off + bytes;
    layout = (layout ^ off) * 1099511628211ull;
    layout = (layout ^ bytes) * 1099511628211ull;
    return reinterpret_cast<void*>(reinterpret_cast<uintptr_t>(base) + off);
  }
};

}  // namespace

struct native_gpu {
  int device = 0;
  int enabled = 0;
  int bf16 = 0;
  int sm_count = 148;
  int debug = 0;
  char device_name[256] = {0};
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  float* d_window = nullptr;
  float2* d_twiddle = nullptr;
  float4* d_rope = nullptr;
  int rope_len = 0;
  // workspace (grow-only)
  long long ws_tokens = 0;
  float* x = nullptr;
  float* x_alt = nullptr;
  void* x16_alt = nullptr;      // sequence parallelism: incoming copies of x16 / row_inv
  float* row_inv_alt = nullptr;
  long long sp_tokens = 0;
  int sp_parity = 0;            // x / x16 / row_inv and their alternates are swapped
  void* x16 = nullptr;          // 16-bit copy of x (A operand of the norm-folded GEMMs)
  float* row_inv = nullptr;     // per-row sqrt(256)/|x| of the current x
  int stats_valid = 0;          // x16 / row_inv describe the current x
  void* qkv = nullptr;
  void* attn = nullptr;
  float* gates = nullptr;
  long long ws_frames = 0;  // segments * frames
  float* spec = nullptr;
  float* mask = nullptr;
  float* frames_buf = nullptr;
  long long ws_seg = 0;     // segments * 2 * segment samples
  float* seg_out = nullptr;
  long long ws_audio = 0;
  float* audio_in = nullptr;
  float* audio_out = nullptr;
  // mask tile tables
  int tiles_frames = 0;
  int4* d_tiles1 = nullptr;
  int n_tiles1 = 0;
  int4* d_tiles2 = nullptr;
  int n_tiles2 = 0;
  // loaded model (vocalarc_b200_load_model)
  int model_loaded = 0;
  int model_from_cache = 0;     // the loaded weights came from a converted image on disk
  uint64_t model_hash = 0;      // content hash of the loaded pack
  void* model_mem = nullptr;
  BlockW blocks[kDepth][2];
  BandW band;
  MaskW maskw;
  // ABI caches
  std::vector<CachedBlock> block_cache;
  void* abi_mask_mem = nullptr;
  uint64_t abi_mask_print = 0;
  int abi_mask_bf16 = -1;
  MaskW abi_mask;
  // resident session of the reference ABI
  int resident_active = 0;
  long long resident_tokens = 0;
  int phys_s = 0, phys_l = 0;   // layout of the device buffer: [phys_s][phys_l]
  int transposed = 0;           // logical layout = [phys_l][phys_s] when set
  // one chunk range of a track sharded across GPUs (vocalarc_b200_range_*)
  int range_ready = 0;          // range_forward completed; finish may run
  int range_length = 0, range_chunk = 0, range_step = 0, range_border = 0, range_plen = 0;
  int range_chunks = 0, range_batch = 1, range_c0 = 0, range_c1 = 0;
  float* seam_out = nullptr;    // partial sums past this range ([3][seam])
  float* seam_in = nullptr;     // the previous range's seam, copied here
  long long seam_cap = 0;       // floats allocated in each seam buffer
  int has_seam_in = 0;
  // The previous range's seam buffer in another process, mapped once per
  // exported handle (opening an IPC mapping costs far more than the copy).
  void* seam_peer = nullptr;
  unsigned char seam_peer_handle[64] = {};
  // bigshift + TTA variant tracks and their estimates (vocalarc_b200_separate_tta)
  long long ws_tta = 0;
  float* tta_in = nullptr;
  float* tta_out = nullptr;
  // host-injected failure (VOCALARC_B200_FAIL_AT=k): the k-th compute call of
  // the C ABI fails as a CUDA error would (0 = off)
  long long fail_at = 0;
  long long abi_calls = 0;
  // launch trace: one event after every launch on the provider stream
  long long launches = 0;
  int trace = 0;
  cudaEvent_t trace_base = nullptr;
  std::vector<cudaEvent_t> event_pool;
  std::vector<std::pair<const char*, cudaEvent_t>> trace_entries;
};

namespace {

bool cuda_ok(native_gpu* g, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "vocalarc-b200: %s failed: %s; falling back to CPU\n", what, cudaGetErrorString(e));
  g->enabled = 0;
  return false;
}

void trace_mark(native_gpu* g, const char* what) {
  const size_t used = g->trace_entries.size();
  if (used == g->event_pool.size()) {
    cudaEvent_t ev = nullptr;
    if (cudaEventCreate(&ev) != cudaSuccess) return;
    g->event_pool.push_back(ev);
  }
  cudaEvent_t ev = g->event_pool[used];
  cudaEventRecord(ev, g->stream);
  g->trace_entries.emplace_back(what, ev);
}

// Counts one compute call of the C ABI.  With VOCALARC_B200_FAIL_AT=k set
// when the provider was created, the k-th such call fails the way a CUDA error
// does (message on stderr, provider disabled, 0 returned), so that a caller's
// fallback can be tested without faulting a GPU.
bool abi_step(native_gpu* g, const char* what) {
  ++g->abi_calls;
  if (g->fail_at <= 0 || g->abi_calls != g->fail_at) return true;
  fprintf(stderr, "vocalarc-b200: %s failed: injected failure (VOCALARC_B200_FAIL_AT=%lld); falling back to CPU\n",
          what, g->fail_at);
  g->enabled = 0;
  return false;
}

bool launched(native_gpu* g, cudaError_t e, const char* what) {
  if (!cuda_ok(g, e, what)) return false;
  ++g->launches;
  if (g->trace) trace_mark(g, what);
  if (g->debug) {
    if (!cuda_ok(g, cudaStreamSynchronize(g->stream), what)) return false;
    int err = 0;
    cudaMemcpy(&err, g->d_err, sizeof(int), cudaMemcpyDeviceToHost);
    fprintf(stderr, "vocalarc-b200: %s ok (device error %d)\n", what, err);
  }
  return true;
}

// Synchronises and turns a recorded device-side wait timeout into a failure.
bool sync_and_check(native_gpu* g, const char* what) {
  if (!cuda_ok(g, cudaStreamSynchronize(g->stream), what)) return false;
  int err = 0;
  if (!cuda_ok(g, cudaMemcpy(&err, g->d_err, sizeof(int), cudaMemcpyDeviceToHost), what)) return false;
  if (err != 0) {
    fprintf(stderr, "vocalarc-b200: %s: kernel gave up waiting (code %d); falling back to CPU\n", what, err);
    cudaMemset(g->d_err, 0, sizeof(int));
    g->enabled = 0;
    return false;
  }
  return true;
}

template <typename P>
bool grow(native_gpu* g, P** ptr, size_t bytes, const char* what) {
  if (*ptr != nullptr) cudaFree(*ptr);
  *ptr = nullptr;
  return cuda_ok(g, cudaMalloc(reinterpret_cast<void**>(ptr), bytes), what);
}

bool ensure_tokens(native_gpu* g, long long tokens) {
  if (tokens <= g->ws_tokens) return true;
  g->ws_tokens = 0;
  const size_t t = static_cast<size_t>(tokens);
  if (!grow(g, &g->x, t * kDim * 4, "cudaMalloc(x)") || !grow(g, &g->x_alt, t * kDim * 4, "cudaMalloc(x_alt)") ||
      !grow(g, &g->x16, t * kDim * 2, "cudaMalloc(x16)") ||
      !grow(g, &g->row_inv, t * 4, "cudaMalloc(row_inv)") ||
      !grow(g, &g->qkv, t * kQkvDim * 2, "cudaMalloc(qkv)") ||
      !grow(g, &g->attn, t * kDimInner * 2, "cudaMalloc(attn)") ||
      !grow(g, &g->gates, t * kHeads * 4, "cudaMalloc(gates)"))
    return false;
  g->ws_tokens = tokens;
  return true;
}

bool ensure_frames(native_gpu* g, long long seg_frames) {
  if (seg_frames <= g->ws_frames) return true;
  g->ws_frames = 0;
  const size_t f = static_cast<size_t>(seg_frames);
  if (!grow(g, &g->spec, f * kFreqBins * 4 * 4, "cudaMalloc(spec)") ||
      !grow(g, &g->mask, f * kFreqBins * 4 * 4, "cudaMalloc(mask)") ||
      !grow(g, &g->frames_buf, f * 2 * kNfft * 4, "cudaMalloc(frames)"))
    return false;
  g->ws_frames = seg_frames;
  return true;
}

bool ensure_seg(native_gpu* g, long long samples) {
  if (samples <= g->ws_seg) return true;
  g->ws_seg = 0;
  if (!grow(g, &g->seg_out, static_cast<size_t>(samples) * 4, "cudaMalloc(seg_out)")) return false;
  g->ws_seg = samples;
  return true;
}

bool ensure_audio(native_gpu* g, long long samples) {
  if (samples <= g->ws_audio) return true;
  g->ws_audio = 0;
  if (!grow(g, &g->audio_in, static_cast<size_t>(samples) * 4, "cudaMalloc(audio_in)") ||
      !grow(g, &g->audio_out, static_cast<size_t>(samples) * 4, "cudaMalloc(audio_out)"))
    return false;
  g->ws_audio = samples;
  return true;
}

// The RoPE cos/sin table (rope_table, apply_rotary's arithmetic) for at least
// `positions` positions.
bool ensure_rope(native_gpu* g, int positions) {
  if (positions <= g->rope_len) return true;
  const int n = positions < 128 ? 128 : positions;
  const std::vector<float4> table = rope_table(n);
  g->rope_len = 0;
  if (!grow(g, &g->d_rope, table.size() * sizeof(float4), "cudaMalloc(rope)")) return false;
  if (!cuda_ok(g, cudaMemcpy(g->d_rope, table.data(), table.size() * sizeof(float4), cudaMemcpyHostToDevice), "rope"))
    return false;
  g->rope_len = n;
  return true;
}

// GEMM operand map: 16-bit [rows][k], box 64 x box_rows, 128-byte swizzle.
bool make_map_rows(native_gpu* g, CUtensorMap* map, const void* base, long long rows, int k, int box_rows) {
  return make_tmap_2d(map, base, 2, static_cast<uint64_t>(k), static_cast<uint64_t>(rows),
                      static_cast<uint64_t>(k) * 2, 64, static_cast<uint32_t>(box_rows), 128, g->bf16 != 0);
}

// Staged-epilogue maps: 16-bit [rows][n] stores in 64 x 32 boxes; fp32 residual
// [rows][256] in 32 x 32 boxes; its 16-bit copy in 32 x 32 boxes (64B swizzle).
bool make_out16_map(native_gpu* g, CUtensorMap* map, const void* base, long long rows, int n) {
  return make_tmap_2d(map, base, 2, static_cast<uint64_t>(n), static_cast<uint64_t>(rows),
                      static_cast<uint64_t>(n) * 2, 64, 32, 128, g->bf16 != 0);
}

// Scales column i of W[out][in] by scale[i] (an RMSNorm gamma folded into the
// GEMM that consumes the norm).
void scale_columns(std::vector<float>& w, int in, const float* scale) {
  const size_t rows = w.size() / static_cast<size_t>(in);
  for (size_t r = 0; r < rows; ++r)
    for (int i = 0; i < in; ++i) w[r * in + i] *= scale[i];
}

// Weight bytes for `dst` (a pointer of `arena`): into the host mirror, or
// straight to the device; nothing in a layout-only pass.
bool put(native_gpu* g, Arena& arena, void* dst, const void* src, size_t bytes, const char* what) {
  if (arena.dry) return true;
  if (arena.host != nullptr) {
    memcpy(arena.host + (reinterpret_cast<uintptr_t>(dst) - reinterpret_cast<uintptr_t>(arena.base)), src, bytes);
    return true;
  }
  return cuda_ok(g, cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), what);
}

bool upload16(native_gpu* g, Arena& arena, const float* packed, int in, int out, void** dst, CUtensorMap* map,
              int box_rows, const float* col_scale = nullptr) {
  *dst = arena.take(static_cast<size_t>(in) * out * 2);
  if (*dst == nullptr) return false;
  if (!arena.dry) {
    std::vector<float> w;
    std::vector<uint16_t> h;
    unpack_packed(packed, in, out, w);
    if (col_scale != nullptr) scale_columns(w, in, col_scale);
    to16(w, g->bf16 != 0, h);
    if (!put(g, arena, *dst, h.data(), h.size() * 2, "upload weight")) return false;
  }
  return !arena.maps || make_map_rows(g, map, *dst, out, in, box_rows);
}

bool upload_f32(native_gpu* g, Arena& arena, const float* src, size_t count, float** dst) {
  *dst = static_cast<float*>(arena.take(count * 4));
  if (*dst == nullptr) return false;
  return put(g, arena, *dst, src, count * 4, "upload vector");
}

constexpr size_t kBlockBytes = (static_cast<size_t>(kQkvRows) * kDim + kDim * kDimInner + 2 * kFfDim * kDim) * 2 +
                               (kHeads + kFfDim + kDim) * 4 + 16 * 1024;

bool upload_block(native_gpu* g, Arena& arena, const native_gpu_transformer_weights& w, BlockW& b) {
  // q|k|v rows, then the gate rows, then zero rows; all scaled by the attention gamma.
  b.qkv = arena.take(static_cast<size_t>(kQkvRows) * kDim * 2);
  if (b.qkv == nullptr) return false;
  if (!arena.dry) {
    std::vector<float> qkv, gw;
    unpack_packed(w.qkv, kDim, kQkvDim, qkv);
    unpack_packed(w.gate_weight, kDim, kHeads, gw);
    qkv.resize(static_cast<size_t>(kQkvRows) * kDim, 0.f);
    std::copy(gw.begin(), gw.end(), qkv.begin() + static_cast<size_t>(kQkvDim) * kDim);
    scale_columns(qkv, kDim, w.gamma);
    std::vector<uint16_t> h;
    to16(qkv, g->bf16 != 0, h);
    if (!put(g, arena, b.qkv, h.data(), h.size() * 2, "qkv")) return false;
  }
  if (arena.maps && !make_map_rows(g, &b.m_qkv, b.qkv, kQkvRows, kDim, 256)) return false;
  if (!upload16(g, arena, w.out_weight, kDimInner, kDim, &b.out, &b.m_out, 256) ||
      !upload16(g, arena, w.ff1_weight, kDim, kFfDim, &b.ff1, &b.m_ff1, 256, w.ff_gamma) ||
      !upload16(g, arena, w.ff2_weight, kFfDim, kDim, &b.ff2, &b.m_ff2, 256))
    return false;
  return upload_f32(g, arena, w.gate_bias, kHeads, &b.gate_b) && upload_f32(g, arena, w.ff1_bias, kFfDim, &b.ff1_b) &&
         upload_f32(g, arena, w.ff2_bias, kDim, &b.ff2_b);
}

int mask_w2_rows_total() {
  int total = 0;
  for (int b = 0; b < kBands; ++b) total += round16(2 * 4 * kBandFreqs[b]);
  return total;
}

constexpr size_t mask_bytes_estimate() {
  return static_cast<size_t>(kBands) * kFfDim * kDim * 2 + kBands * kFfDim * 4 + 8400ull * kFfDim * 2 + 8400 * 4 +
         kDim * 4 + 256 * 1024;
}

// Mask head weights: first layers stacked [90*1024][256]; second layers with
// rows interleaved (value i, gate i) so the GLU pairs are adjacent columns,
// each band padded to a multiple of 16 rows.
// Bands [band_lo, band_hi) are converted (the layout is always the whole head,
// so several calls over one arena can split the work); write_bias also
// converts the bias vectors.
bool upload_mask(native_gpu* g, Arena& arena, const native_gpu_mask_band* bands, const float* final_gamma, MaskW& m,
                 int band_lo = 0, int band_hi = kBands, bool write_bias = true) {
  const bool bf = g->bf16 != 0;
  int off = 0;
  for (int b = 0; b < kBands; ++b) {
    m.w2_off[b] = off;
    m.w2_rows[b] = round16(2 * bands[b].input_dim);
    off += m.w2_rows[b];
  }
  m.w2_total = off;
  std::vector<float> w, rows, bias;
  std::vector<uint16_t> h;
  // Layer 1, band by band: [1024][256] with the final RMSNorm gamma folded.
  const size_t w1_band = static_cast<size_t>(kFfDim) * kDim;
  m.w1 = arena.take(kBands * w1_band * 2);
  if (m.w1 == nullptr) return false;
  if (!arena.dry) {
    bias.resize(static_cast<size_t>(kBands) * kFfDim);
    for (int b = 0; b < kBands; ++b) memcpy(&bias[static_cast<size_t>(b) * kFfDim], bands[b].first_bias, kFfDim * 4);
    for (int b = band_lo; b < band_hi; ++b) {
      unpack_packed(bands[b].first_weight, kDim, kFfDim, w);
      scale_columns(w, kDim, final_gamma);
      to16(w, bf, h);
      if (!put(g, arena, static_cast<char*>(m.w1) + b * w1_band * 2, h.data(), w1_band * 2, "mask w1")) return false;
    }
  }
  if (arena.maps && !make_map_rows(g, &m.m_w1, m.w1, static_cast<long long>(kBands) * kFfDim, kDim, 256)) return false;
  m.b1 = static_cast<float*>(arena.take(static_cast<size_t>(kBands) * kFfDim * 4));
  if (m.b1 == nullptr || (write_bias && !put(g, arena, m.b1, bias.data(), bias.size() * 4, "mask b1"))) return false;
  // Layer 2, band by band: rows interleaved (value i, gate i), zero rows up to a multiple of 16.
  m.w2 = arena.take(static_cast<size_t>(m.w2_total) * kFfDim * 2);
  if (m.w2 == nullptr) return false;
  if (!arena.dry) {
    bias.assign(m.w2_total, 0.f);
    for (int b = 0; b < kBands; ++b)
      for (int i = 0; i < bands[b].input_dim; ++i) {
        bias[m.w2_off[b] + 2 * i] = bands[b].second_bias[i];
        bias[m.w2_off[b] + 2 * i + 1] = bands[b].second_bias[bands[b].input_dim + i];
      }
    for (int b = band_lo; b < band_hi; ++b) {
      const int d = bands[b].input_dim;
      const int o = m.w2_off[b];
      unpack_packed(bands[b].second_weight, kFfDim, 2 * d, w);
      rows.assign(static_cast<size_t>(m.w2_rows[b]) * kFfDim, 0.f);
      for (int i = 0; i < d; ++i) {
        memcpy(&rows[static_cast<size_t>(2 * i) * kFfDim], &w[static_cast<size_t>(i) * kFfDim], kFfDim * 4);
        memcpy(&rows[static_cast<size_t>(2 * i + 1) * kFfDim], &w[static_cast<size_t>(d + i) * kFfDim], kFfDim * 4);
      }
      to16(rows, bf, h);
      if (!put(g, arena, static_cast<char*>(m.w2) + static_cast<size_t>(o) * kFfDim * 2, h.data(), h.size() * 2,
               "mask w2"))
        return false;
    }
  }
  if (arena.maps && !make_map_rows(g, &m.m_w2, m.w2, m.w2_total, kFfDim, 16)) return false;
  m.b2 = static_cast<float*>(arena.take(static_cast<size_t>(m.w2_total) * 4));
  return m.b2 != nullptr && (!write_bias || put(g, arena, m.b2, bias.data(), bias.size() * 4, "mask b2"));
}

bool ensure_mask_tiles(native_gpu* g, int frames, const MaskW& m) {
  if (g->tiles_frames == frames && g->d_tiles1 != nullptr) return true;
  std::vector<int4> t1, t2;
  for (int b = 0; b < kBands; ++b)
    for (int m0 = 0; m0 < frames; m0 += 128) {
      const int mv = frames - m0 < 128 ? frames - m0 : 128;
      for (int n0 = 0; n0 < kFfDim; n0 += 256) t1.push_back(make_tile(b * frames + m0, b * kFfDim + n0, n0, mv, 256, b));
      for (int n0 = 0; n0 < m.w2_rows[b]; n0 += 256) {
        const int ns = m.w2_rows[b] - n0 < 256 ? m.w2_rows[b] - n0 : 256;
        t2.push_back(make_tile(b * frames + m0, m.w2_off[b] + n0, n0, mv, ns, b));
      }
    }
  g->tiles_frames = 0;
  if (!grow(g, &g->d_tiles1, t1.size() * sizeof(int4), "cudaMalloc(tiles)") ||
      !grow(g, &g->d_tiles2, t2.size() * sizeof(int4), "cudaMalloc(tiles)"))
    return false;
  if (!cuda_ok(g, cudaMemcpy(g->d_tiles1, t1.data(), t1.size() * sizeof(int4), cudaMemcpyHostToDevice), "tiles") ||
      !cuda_ok(g, cudaMemcpy(g->d_tiles2, t2.data(), t2.size() * sizeof(int4), cudaMemcpyHostToDevice), "tiles"))
    return false;
  g->n_tiles1 = static_cast<int>(t1.size());
  g->n_tiles2 = static_cast<int>(t2.size());
  g->tiles_frames = frames;
  return true;
}

GemmArgs uniform_args(native_gpu* g, long long rows, int n, int k) {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.m_rows = static_cast<int>(rows);
  a.n_tiles = n / 256;
  a.k_blocks = k / 64;
  a.num_tiles = static_cast<int>((rows + 127) / 128) * a.n_tiles;
  a.err = g->d_err;
  a.pos_div = 1;
  a.pos_mod = 1;
  return a;
}

// ------------------------------------------------------------------ one axial block

bool ensure_stats(native_gpu* g, long long tokens, int remap_s0 = 0, int remap_l0 = 0) {
  if (g->stats_valid && remap_s0 == 0) return true;
  if (!launched(g, launch_row_stats(g->x, tokens, g->x16, g->row_inv, g->bf16 != 0, remap_s0, remap_l0, g->stream),
                "row stats"))
    return false;
  g->stats_valid = remap_s0 == 0;
  return true;
}

bool provider_hook(void* owner, cudaError_t e, const char* what) {
  return launched(static_cast<native_gpu*>(owner), e, what);
}

// One axial block on the residual stream g->x (transformer_forward,
// vocalarc_separation.c:836-873) through the shared orchestration of
// block.cu.  Needs x16 / row_inv of the current x; leaves them valid for the
// updated x.
bool run_block(native_gpu* g, const BlockW& w, long long tokens, const AxisPlan& ax) {
  if (!ensure_rope(g, ax.length) || !ensure_stats(g, tokens)) return false;
  const AxialBuffers buf{g->x,     g->x16,    g->row_inv, nullptr,     g->qkv,
                         g->attn,  g->gates,  g->d_rope,  g->d_err,    g->rope_len};
  const AxialWeights aw{&w.m_qkv, &w.m_out, &w.m_ff1, &w.m_ff2, w.ff1, w.gate_b, w.ff1_b, w.ff2_b};
  if (!run_axial_block(buf, aw, AxialShape{kDim, kFfDim, 0}, tokens, ax, g->bf16 != 0, g->sm_count, g->stream,
                       provider_hook, g))
    return false;
  g->stats_valid = 1;
  return true;
}

// Final RMSNorm (gamma folded into the first mask layer) + mask MLPs over
// `segments` x 90 x frames band-major tokens.  frame_major_rows: the physical
// rows are [frames][90] and the row statistics are written band-major.
bool run_mask(native_gpu* g, const MaskW& m, int segments, int frames, bool frame_major_rows, bool ref_layout,
              float* mask_out) {
  const bool bf = g->bf16 != 0;
  const long long tokens = static_cast<long long>(segments) * kBands * frames;
  if (!ensure_stats(g, tokens, frame_major_rows ? frames : 0, frame_major_rows ? kBands : 0)) return false;
  if (!ensure_mask_tiles(g, frames, m)) return false;
  GemmMaps maps;
  if (!make_map_rows(g, &maps.a, g->x16, tokens, kDim, 128)) return false;
  maps.b = m.m_w1;
  maps.c = maps.d = maps.a;
  GemmArgs args;
  memset(&args, 0, sizeof(args));
  args.k_blocks = kDim / 64;
  args.tiles = g->d_tiles1;
  args.tiles_per_chunk = g->n_tiles1;
  args.chunk_rows = kBands * frames;
  args.num_tiles = g->n_tiles1 * segments;
  args.out = g->qkv;
  args.ldo = kFfDim;
  args.bias = m.b1;
  args.row_inv = g->row_inv;
  args.err = g->d_err;
  args.pos_div = args.pos_mod = 1;
  if (!launched(g, launch_gemm(kEpiTanhBand, bf, maps, args, g->sm_count, g->stream), "mask gemm 1")) return false;
  if (!make_map_rows(g, &maps.a, g->qkv, tokens, kFfDim, 128)) return false;
  maps.b = m.m_w2;
  args.k_blocks = kFfDim / 64;
  args.tiles = g->d_tiles2;
  args.tiles_per_chunk = g->n_tiles2;
  args.num_tiles = g->n_tiles2 * segments;
  args.b_box16 = 1;
  args.out = mask_out;
  args.ldo = 0;
  args.bias = m.b2;
  args.row_inv = nullptr;
  args.frames = frames;
  args.mask_ref_layout = ref_layout ? 1 : 0;
  return launched(g, launch_gemm(kEpiGluMask, bf, maps, args, g->sm_count, g->stream), "mask gemm 2");
}

AxisPlan time_axis(int segments, int frames) {
  return AxisPlan{1, frames, kBands, segments, segments * kBands, frames, 1, frames};
}
AxisPlan band_axis(int segments, int frames) {
  return AxisPlan{2, frames, kBands, segments, segments * frames, kBands, frames, kBands};
}

// Full forward of `segments` equal-length segments (T frames each).
bool forward_segments(native_gpu* g, const float* d_audio, const SegmentMap& map, int segments, int frames,
                      float* d_seg_out) {
  const long long tokens = static_cast<long long>(segments) * kBands * frames;
  if (!ensure_tokens(g, tokens) || !ensure_frames(g, static_cast<long long>(segments) * frames)) return false;
  if (!launched(g, launch_stft(d_audio, map, segments, frames, g->d_window, g->d_twiddle, g->spec, g->stream), "stft"))
    return false;
  if (!launched(g, launch_band_split(g->spec, segments, frames, g->band.wt, g->band.wt_off, g->band.gamma,
                                     g->band.gamma_off, g->band.bias, g->x, g->stream),
                "band split"))
    return false;
  g->stats_valid = 0;
  for (int layer = 0; layer < kDepth; ++layer) {
    if (!run_block(g, g->blocks[layer][0], tokens, time_axis(segments, frames))) return false;
    if (!run_block(g, g->blocks[layer][1], tokens, band_axis(segments, frames))) return false;
  }
  if (!run_mask(g, g->maskw, segments, frames, false, false, g->mask)) return false;
  if (!launched(g, launch_istft_frames(g->spec, g->mask, segments, frames, g->d_window, g->d_twiddle, g->frames_buf,
                                       g->stream),
                "istft"))
    return false;
  return launched(g, launch_overlap_add(g->frames_buf, segments, frames, map.seg_length, g->d_window, d_seg_out,
                                        g->stream),
                  "overlap-add");
}

// Largest number of chunk-sized segments that fit comfortably in free memory.
int max_segments(native_gpu* g, int frames, int seg_length) {
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess) return 1;
  const double per_token = kDim * 4.0 * 2 + kDim * 2 + kQkvDim * 2 + kDimInner * 2 + kHeads * 4;
  const double per_seg = per_token * kBands * frames + frames * (kFreqBins * 32.0 + 2 * kNfft * 4.0) +
                         2.0 * seg_length * 4;
  // Count what is already allocated as available for reuse.
  const double have = g->ws_tokens * per_token;
  const double budget = (static_cast<double>(free_b) + have) * 0.7 - 512.0 * 1024 * 1024;
  int n = static_cast<int>(budget / per_seg);
  if (n < 1) n = 1;
  if (n > 64) n = 64;
  return n;
}

bool separate_device_impl(native_gpu* g, const float* d_audio, int tracks, int length, int chunked, int chunk_samples,
                          int model_batch, float* d_vocals) {
  if (!g->model_loaded) {
    fprintf(stderr, "vocalarc-b200: no model loaded (vocalarc_b200_load_model)\n");
    return false;
  }
  if (length <= 0 || tracks <= 0) return false;
  if (!chunked) {
    const int frames = length / kHop + 1;
    const int per_pass = max_segments(g, frames, length);
    for (int t0 = 0; t0 < tracks; t0 += per_pass) {
      const int n = tracks - t0 < per_pass ? tracks - t0 : per_pass;
      const SegmentMap map = whole_clip_map(length);
      // Whole clips write their overlap-add output straight into the vocals buffer.
      if (!forward_segments(g, d_audio + static_cast<long long>(t0) * 2 * length, map, n, frames,
                            d_vocals + static_cast<long long>(t0) * 2 * length))
        return false;
    }
    return true;
  }
  const int chunk = chunk_samples > 0 ? chunk_samples : 881559;
  const int step = chunk / 2;
  const int border = chunk - step;
  const bool padded = length > 2 * border && border > 0;
  const int plen = padded ? length + 2 * border : length;
  const int chunks = (plen + step - 1) / step;
  const int frames = chunk / kHop + 1;
  if (model_batch < 1) model_batch = 1;
  if (!ensure_seg(g, static_cast<long long>(chunks) * 2 * chunk)) return false;
  const int per_pass = max_segments(g, frames, chunk);
  for (int tr = 0; tr < tracks; ++tr) {
    const float* audio = d_audio + static_cast<long long>(tr) * 2 * length;
    for (int c0 = 0; c0 < chunks; c0 += per_pass) {
      const int n = chunks - c0 < per_pass ? chunks - c0 : per_pass;
      const SegmentMap mm = demix_map(length, chunk, padded ? border : 0, plen, step, c0);
      if (!forward_segments(g, audio, mm, n, frames, g->seg_out + static_cast<long long>(c0) * 2 * chunk)) return false;
    }
    const SegmentMap dm = demix_map(length, chunk, padded ? border : 0, plen, step, 0);
    if (!launched(g, launch_demix(g->seg_out, dm, chunks, model_batch,
                                  d_vocals + static_cast<long long>(tr) * 2 * length, g->stream),
                  "demix"))
      return false;
  }
  return true;
}

// ------------------------------------------------------------------ sequence parallelism
// One clip's whole-clip forward split across providers (one per GPU): rank r
// holds the band range [kBands r / n, kBands (r + 1) / n) over all T frames for
// the time-axis blocks (band-major [nb][T] rows), and the frame range
// [T s / n, T (s + 1) / n) over all 90 bands for the band-axis blocks
// ([90][nf] rows).  Between axes every rank copies to every other the rows the
// other needs -- x, its 16-bit copy and the row RMSNorm factor, so the row
// statistics stay valid and every row sees exactly the arithmetic of the
// single-GPU forward.  A copy is one 2-D block (rows of one band are
// contiguous in both layouts).
struct SpCopy {
  int src, dst;
  long long src_row, src_pitch, dst_row, dst_pitch, width, height;   // in token rows
};

int sp_band_lo(int r, int n) { return kBands * r / n; }
int sp_frame_lo(int r, int n, int frames) { return static_cast<int>(static_cast<long long>(frames) * r / n); }

// Phase 0: rank 0's full band-major x to the other ranks' band ranges.
// Phase 1: band ranges -> frame ranges.  Phase 2: frame ranges -> band ranges.
// Phase 3: frame ranges -> rank 0's full band-major x.
std::vector<SpCopy> sp_plan(int n, int frames, int phase) {
  std::vector<SpCopy> plan;
  const long long t = frames;
  for (int d = 0; d < n; ++d)
    for (int r = 0; r < n; ++r) {
      const long long nb_d = sp_band_lo(d + 1, n) - sp_band_lo(d, n), nb_r = sp_band_lo(r + 1, n) - sp_band_lo(r, n);
      const long long nf_d = sp_frame_lo(d + 1, n, frames) - sp_frame_lo(d, n, frames);
      const long long nf_r = sp_frame_lo(r + 1, n, frames) - sp_frame_lo(r, n, frames);
      SpCopy c{r, d, 0, 0, 0, 0, 0, 0};
      if (phase == 0) {
        if (r != 0 || d == 0) continue;
        c = SpCopy{0, d, sp_band_lo(d, n) * t, nb_d * t, 0, nb_d * t, nb_d * t, 1};
      } else if (phase == 1) {
        c = SpCopy{r, d, sp_frame_lo(d, n, frames), t, sp_band_lo(r, n) * nf_d, nf_d, nf_d, nb_r};
      } else if (phase == 2) {
        c = SpCopy{r, d, sp_band_lo(d, n) * nf_r, nf_r, sp_frame_lo(r, n, frames), t, nf_r, nb_d};
      } else {
        if (d != 0) continue;
        c = SpCopy{r, 0, 0, nf_r, sp_frame_lo(r, n, frames), t, nf_r, kBands};
      }
      if (c.width > 0 && c.height > 0) plan.push_back(c);
    }
  return plan;
}

void sp_swap(native_gpu* g) {
  std::swap(g->x, g->x_alt);
  std::swap(g->x16, g->x16_alt);
  std::swap(g->row_inv, g->row_inv_alt);
  g->sp_parity ^= 1;
}

// Workspace for rows of every layout plus the alternates the copies land in.
bool ensure_sp(native_gpu* g, long long tokens) {
  if (g->sp_parity) sp_swap(g);
  if (!ensure_tokens(g, tokens)) return false;
  if (tokens <= g->sp_tokens) return true;
  g->sp_tokens = 0;
  if (!grow(g, &g->x16_alt, static_cast<size_t>(tokens) * kDim * 2, "cudaMalloc(x16_alt)") ||
      !grow(g, &g->row_inv_alt, static_cast<size_t>(tokens) * 4, "cudaMalloc(row_inv_alt)"))
    return false;
  g->sp_tokens = tokens;
  return true;
}

// One exchange: each destination's stream waits for every source's last
// block (ev), then copies x, x16 and row_inv.  Phase 0 writes straight into
// the destination's buffers; the others write into its alternates, which it
// then swaps in.  Source pointers are taken before any swap of this phase.
bool sp_exchange(native_gpu* const* gpus, int n, int frames, int phase, const std::vector<cudaEvent_t>& ev) {
  std::vector<float*> sx(n), sinv(n);
  std::vector<char*> s16(n);
  for (int r = 0; r < n; ++r) {
    sx[r] = gpus[r]->x;
    s16[r] = static_cast<char*>(gpus[r]->x16);
    sinv[r] = gpus[r]->row_inv;
  }
  const std::vector<SpCopy> plan = sp_plan(n, frames, phase);
  for (int d = 0; d < n; ++d) {
    native_gpu* g = gpus[d];
    bool any = false;
    for (const SpCopy& c : plan) any = any || c.dst == d;
    if (!any) continue;
    cudaSetDevice(g->device);
    for (int r = 0; r < n; ++r)
      if (r != d && !cuda_ok(g, cudaStreamWaitEvent(g->stream, ev[r], 0), "exchange wait")) return false;
    float* dx = phase == 0 ? g->x : g->x_alt;
    char* d16 = static_cast<char*>(phase == 0 ? g->x16 : g->x16_alt);
    float* dinv = phase == 0 ? g->row_inv : g->row_inv_alt;
    for (const SpCopy& c : plan) {
      if (c.dst != d) continue;
      const size_t rx = kDim * 4, r16 = kDim * 2, ri = 4;
      if (!cuda_ok(g, cudaMemcpy2DAsync(reinterpret_cast<char*>(dx) + c.dst_row * rx, c.dst_pitch * rx,
                                        reinterpret_cast<const char*>(sx[c.src]) + c.src_row * rx, c.src_pitch * rx,
                                        c.width * rx, c.height, cudaMemcpyDefault, g->stream),
                   "exchange x") ||
          !cuda_ok(g, cudaMemcpy2DAsync(d16 + c.dst_row * r16, c.dst_pitch * r16, s16[c.src] + c.src_row * r16,
                                        c.src_pitch * r16, c.width * r16, c.height, cudaMemcpyDefault, g->stream),
                   "exchange x16") ||
          !cuda_ok(g, cudaMemcpy2DAsync(reinterpret_cast<char*>(dinv) + c.dst_row * ri, c.dst_pitch * ri,
                                        reinterpret_cast<const char*>(sinv[c.src]) + c.src_row * ri,
                                        c.src_pitch * ri, c.width * ri, c.height, cudaMemcpyDefault, g->stream),
                   "exchange row factor"))
        return false;
    }
    if (phase != 0) sp_swap(g);
    g->stats_valid = 1;
  }
  return true;
}

struct PackCursor {
  const unsigned char* p;
  const unsigned char* end;
  const float* next(uint64_t expected) {
    if (static_cast<size_t>(end - p) < 8) return nullptr;
    uint64_t count;
    memcpy(&count, p, 8);
    p += 8;
    if (count != expected || static_cast<size_t>(end - p) < count * 4) return nullptr;
    const float* r = reinterpret_cast<const float*>(p);
    p += count * 4;
    return r;
  }
};

// Tensor pointers of one VSCNAT01 pack (model_parse, vocalarc_separation.c:528-589).
struct PackView {
  native_gpu_transformer_weights layers[kDepth][2];
  const float* bg[kBands];
  const float* bw[kBands];
  const float* bb[kBands];
  const float* final_gamma = nullptr;
  native_gpu_mask_band mb[kBands];
};

bool parse_pack_view(const void* pack, size_t bytes, PackView& v) {
  if (pack == nullptr || bytes < 64) return false;
  const unsigned char* base = static_cast<const unsigned char*>(pack);
  uint32_t fields[14];
  memcpy(fields, base + 8, sizeof(fields));
  const uint32_t expect[12] = {1, kDim, kDepth, kBands, kHeads, kDimHead, kFreqBins, kChannels, kNfft, kHop, kNfft,
                               kModelFrames};
  if (memcmp(base, "VSCNAT01", 8) != 0 || memcmp(fields, expect, sizeof(expect)) != 0) {
    fprintf(stderr, "vocalarc-b200: unsupported native model header\n");
    return false;
  }
  PackCursor cur{base + 64, base + bytes};
  for (int l = 0; l < kDepth; ++l)
    for (int a = 0; a < 2; ++a) {
      native_gpu_transformer_weights& w = v.layers[l][a];
      w.gamma = cur.next(kDim);
      w.qkv = cur.next(static_cast<uint64_t>(kQkvDim) * kDim);
      w.gate_weight = cur.next(kHeads * kDim);
      w.gate_bias = cur.next(kHeads);
      w.out_weight = cur.next(static_cast<uint64_t>(kDim) * kDimInner);
      w.ff_gamma = cur.next(kDim);
      w.ff1_weight = cur.next(static_cast<uint64_t>(kFfDim) * kDim);
      w.ff1_bias = cur.next(kFfDim);
      w.ff2_weight = cur.next(static_cast<uint64_t>(kDim) * kFfDim);
      w.ff2_bias = cur.next(kDim);
      if (!w.gamma || !w.qkv || !w.gate_weight || !w.gate_bias || !w.out_weight || !w.ff_gamma || !w.ff1_weight ||
          !w.ff1_bias || !w.ff2_weight || !w.ff2_bias) {
        fprintf(stderr, "vocalarc-b200: native model truncated in layer %d\n", l);
        return false;
      }
    }
  for (int b = 0; b < kBands; ++b) {
    const int d = 4 * kBandFreqs[b];
    v.bg[b] = cur.next(d);
    v.bw[b] = cur.next(static_cast<uint64_t>(kDim) * d);
    v.bb[b] = cur.next(kDim);
    if (!v.bg[b] || !v.bw[b] || !v.bb[b]) return false;
  }
  v.final_gamma = cur.next(kDim);
  if (v.final_gamma == nullptr) return false;
  for (int b = 0; b < kBands; ++b) {
    const int d = 4 * kBandFreqs[b];
    v.mb[b].first_weight = cur.next(static_cast<uint64_t>(kFfDim) * kDim);
    v.mb[b].first_bias = cur.next(kFfDim);
    v.mb[b].second_weight = cur.next(static_cast<uint64_t>(2 * d) * kFfDim);
    v.mb[b].second_bias = cur.next(2 * d);
    v.mb[b].input_dim = d;
    v.mb[b].first_frequency = band_first(b);
    if (!v.mb[b].first_weight || !v.mb[b].first_bias || !v.mb[b].second_weight || !v.mb[b].second_bias) return false;
  }
  return true;
}

// Band split for the SIMT kernel: W^T per band ([d_b][256]), gammas in bin
// order, biases [90][256], and the two offset tables.
bool upload_band(native_gpu* g, Arena& arena, const PackView& v, BandW& out) {
  std::vector<long long> wt_off(kBands);
  std::vector<int> g_off(kBands + 1);
  size_t cur_wt = 0;
  int cur_g = 0;
  for (int b = 0; b < kBands; ++b) {
    const int d = 4 * kBandFreqs[b];
    wt_off[b] = static_cast<long long>(cur_wt);
    cur_wt += static_cast<size_t>(d) * kDim;
    g_off[b] = cur_g;
    cur_g += d;
  }
  g_off[kBands] = cur_g;
  std::vector<float> wt, gam, bias, w;
  if (!arena.dry) {
    wt.resize(static_cast<size_t>(kBandSplitDim) * kDim);
    gam.resize(kBandSplitDim);
    bias.resize(static_cast<size_t>(kBands) * kDim);
    for (int b = 0; b < kBands; ++b) {
      const int d = 4 * kBandFreqs[b];
      unpack_packed(v.bw[b], d, kDim, w);  // w[n][k]
      for (int k = 0; k < d; ++k)
        for (int n = 0; n < kDim; ++n)
          wt[static_cast<size_t>(wt_off[b]) + static_cast<size_t>(k) * kDim + n] = w[static_cast<size_t>(n) * d + k];
      memcpy(&gam[g_off[b]], v.bg[b], d * 4);
      memcpy(&bias[static_cast<size_t>(b) * kDim], v.bb[b], kDim * 4);
    }
  }
  if (!upload_f32(g, arena, wt.data(), static_cast<size_t>(kBandSplitDim) * kDim, &out.wt) ||
      !upload_f32(g, arena, gam.data(), kBandSplitDim, &out.gamma) ||
      !upload_f32(g, arena, bias.data(), static_cast<size_t>(kBands) * kDim, &out.bias))
    return false;
  out.wt_off = static_cast<long long*>(arena.take(kBands * 8));
  if (out.wt_off == nullptr || !put(g, arena, out.wt_off, wt_off.data(), kBands * 8, "band offsets")) return false;
  out.gamma_off = static_cast<int*>(arena.take((kBands + 1) * 4));
  return out.gamma_off != nullptr && put(g, arena, out.gamma_off, g_off.data(), (kBands + 1) * 4, "band offsets");
}

// ------------------------------------------------------------------ model image
// The loaded model is one device allocation split into fixed regions: one per
// axial block, then the band split, then the mask head.  A region is filled
// by one task, so the tasks run on separate threads into a host image that
// reaches the device in a single copy, and that image can be kept on disk.
constexpr size_t round4k(size_t x) { return (x + 4095) & ~size_t(4095); }
constexpr size_t kBandBytes = static_cast<size_t>(kBandSplitDim) * kDim * 4 + kBandSplitDim * 4 +
                              static_cast<size_t>(kBands) * kDim * 4 + kBands * 8 + (kBands + 1) * 4 + 16 * 1024;
constexpr size_t kBlockRegion = round4k(kBlockBytes);
constexpr size_t kBandRegion = round4k(kBandBytes);
constexpr size_t kMaskRegion = round4k(mask_bytes_estimate());
constexpr int kMaskTasks = 6;   // the mask head's conversion is split by bands over this many tasks
constexpr int kModelTasks = 2 * kDepth + 1 + kMaskTasks;
constexpr size_t kModelBytes = 2 * kDepth * kBlockRegion + kBandRegion + kMaskRegion;

size_t task_offset(int t) {
  if (t < 2 * kDepth) return static_cast<size_t>(t) * kBlockRegion;
  return 2 * kDepth * kBlockRegion + (t == 2 * kDepth ? 0 : kBandRegion);
}
size_t task_size(int t) { return t < 2 * kDepth ? kBlockRegion : (t == 2 * kDepth ? kBandRegion : kMaskRegion); }

// Task t: axial block (t / 2, t % 2) for t < 32, 32 = band split, 33.. = mask
// head, each of those converting a sixth of the bands in the same region.
bool model_task(native_gpu* g, const PackView& v, int t, char* base, uint8_t* host, bool dry, bool maps,
                BlockW (&blocks)[kDepth][2], BandW& band, MaskW& mask, uint64_t* layout) {
  Arena a;
  a.base = reinterpret_cast<char*>(reinterpret_cast<uintptr_t>(base) + task_offset(t));
  a.cap = task_size(t);
  a.host = host != nullptr ? host + task_offset(t) : nullptr;
  a.dry = dry;
  a.maps = maps;
  bool ok;
  if (t < 2 * kDepth)
    ok = upload_block(g, a, v.layers[t / 2][t % 2], blocks[t / 2][t % 2]);
  else if (t == 2 * kDepth)
    ok = upload_band(g, a, v, band);
  else {
    const int k = t - (2 * kDepth + 1);
    ok = upload_mask(g, a, v.mb, v.final_gamma, mask, kBands * k / kMaskTasks, kBands * (k + 1) / kMaskTasks, k == 0);
  }
  *layout = a.layout;
  return ok;
}

uint64_t fold_layout(const uint64_t* h) {
  uint64_t r = 1469598103934665603ull ^ kModelBytes;
  for (int t = 0; t < kModelTasks; ++t) {
    r = (r ^ h[t]) * 1099511628211ull;
    r = (r ^ task_offset(t)) * 1099511628211ull;
  }
  return r;
}

// Nominal device base for host-only conversion: pointers there only locate
// bytes in the image, and a null base would make the first one look like a
// failed allocation.
char* const kHostOnlyBase = reinterpret_cast<char*>(uintptr_t(1) << 20);

int load_threads() {
  const char* v = getenv("VOCALARC_B200_LOAD_THREADS");
  if (v != nullptr && atoi(v) > 0) return atoi(v);
  const unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 4 : (n > 16 ? 16 : static_cast<int>(n));
}

// Converts every region into `image` (kModelBytes, zero-filled by the caller)
// on `threads` threads; `layout` is the fold of the regions' layout hashes.
bool build_image(native_gpu* g, const PackView& v, char* base, uint8_t* image, int threads, uint64_t* layout) {
  uint64_t h[kModelTasks] = {};
  // The mask head's tasks and the band split are the largest: start them first.
  int order[kModelTasks];
  int n_order = 0;
  for (int t = 2 * kDepth + 1; t < kModelTasks; ++t) order[n_order++] = t;
  order[n_order++] = 2 * kDepth;
  for (int t = 0; t < 2 * kDepth; ++t) order[n_order++] = t;
  std::atomic<int> next{0};
  std::atomic<bool> ok{true};
  auto worker = [&]() {
    // Pointers land in scratch copies (equal to the layout pass's); no tensor maps.
    std::vector<BlockW> scratch(2 * kDepth);
    BlockW(*blocks)[kDepth][2] = reinterpret_cast<BlockW(*)[kDepth][2]>(scratch.data());
    BandW band;
    MaskW mask;
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= kModelTasks) break;
      const int t = order[i];
      if (!model_task(g, v, t, base, image, false, false, *blocks, band, mask, &h[t])) ok = false;
    }
  };
  const int n = threads < 1 ? 1 : (threads > kModelTasks ? kModelTasks : threads);
  std::vector<std::thread> pool;
  for (int i = 1; i < n; ++i) pool.emplace_back(worker);
  worker();
  for (auto& th : pool) th.join();
  *layout = fold_layout(h);
  return ok.load();
}

// 64-bit hash of the pack bytes (four interleaved multiply-xorshift lanes).
uint64_t content_hash(const void* p, size_t n) {
  const unsigned char* c = static_cast<const unsigned char*>(p);
  uint64_t lane[4] = {0x9E3779B97F4A7C15ull ^ n, 0xC2B2AE3D27D4EB4Full, 0x165667B19E3779F9ull, 0xD6E8FEB86659FD93ull};
  size_t i = 0;
  for (; i + 32 <= n; i += 32)
    for (int k = 0; k < 4; ++k) {
      uint64_t w;
      memcpy(&w, c + i + 8 * k, 8);
      lane[k] = (lane[k] ^ w) * 0xFF51AFD7ED558CCDull;
      lane[k] ^= lane[k] >> 29;
    }
  uint64_t h = lane[0] ^ (lane[1] * 31) ^ (lane[2] * 961) ^ (lane[3] * 29791);
  for (; i < n; ++i) h = (h ^ c[i]) * 1099511628211ull;
  h ^= h >> 33;
  h *= 0xFF51AFD7ED558CCDull;
  return h ^ (h >> 33);
}

// On-disk image: this header, then kModelBytes of the device arena.
struct ImageHeader {
  char magic[8];
  uint64_t pack_hash;
  uint64_t pack_bytes;
  uint64_t layout_hash;
  uint64_t image_bytes;
  uint64_t image_hash;   // content_hash of the image bytes, checked before use
  uint32_t bf16;
  uint32_t reserved[3];
};
static_assert(sizeof(ImageHeader) == 64, "image header is 64 bytes");

ImageHeader image_header(uint64_t pack_hash, size_t pack_bytes, uint64_t layout, int bf16) {
  ImageHeader h;
  memset(&h, 0, sizeof(h));
  memcpy(h.magic, "VBIMG001", 8);
  h.pack_hash = pack_hash;
  h.pack_bytes = pack_bytes;
  h.layout_hash = layout;
  h.image_bytes = kModelBytes;
  h.bf16 = bf16 ? 1u : 0u;
  return h;
}

// Directory of converted images: VOCALARC_B200_IMAGE_CACHE ("off" disables),
// else $XDG_CACHE_HOME/vocalarc-b200, else $HOME/.cache/vocalarc-b200.
std::string image_cache_dir() {
  const char* v = getenv("VOCALARC_B200_IMAGE_CACHE");
  if (v != nullptr) {
    if (*v == 0 || strcmp(v, "off") == 0 || strcmp(v, "0") == 0) return "";
    return v;
  }
  const char* x = getenv("XDG_CACHE_HOME");
  if (x != nullptr && *x != 0) return std::string(x) + "/vocalarc-b200";
  const char* home = getenv("HOME");
  if (home != nullptr && *home != 0) return std::string(home) + "/.cache/vocalarc-b200";
  return "";
}

std::string image_path(const std::string& dir, const ImageHeader& h) {
  char name[64];
  snprintf(name, sizeof(name), "/%016llx.%s.vbimg", static_cast<unsigned long long>(h.pack_hash),
           h.bf16 ? "bf16" : "fp16");
  return dir + name;
}

bool make_dirs(const std::string& dir) {
  for (size_t i = 1; i <= dir.size(); ++i) {
    if (i == dir.size() || dir[i] == '/') {
      const std::string part = dir.substr(0, i);
      if (mkdir(part.c_str(), 0755) != 0 && errno != EEXIST) return false;
    }
  }
  return true;
}

// The cached image at `path` when its header matches `want` (all but the
// image hash) and its bytes hash to the recorded value; nullptr otherwise.
const uint8_t* map_image(const std::string& path, const ImageHeader& want, size_t* mapped) {
  const int fd = open(path.c_str(), O_RDONLY);
  if (fd < 0) return nullptr;
  struct stat st;
  if (fstat(fd, &st) != 0 || static_cast<size_t>(st.st_size) != sizeof(ImageHeader) + want.image_bytes) {
    close(fd);
    return nullptr;
  }
  void* m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return nullptr;
  ImageHeader have;
  memcpy(&have, m, sizeof(have));
  ImageHeader expect = want;
  expect.image_hash = have.image_hash;
  if (memcmp(&have, &expect, sizeof(ImageHeader)) != 0 ||
      content_hash(static_cast<const uint8_t*>(m) + sizeof(ImageHeader), want.image_bytes) != have.image_hash) {
    munmap(m, static_cast<size_t>(st.st_size));
    return nullptr;
  }
  *mapped = static_cast<size_t>(st.st_size);
  return static_cast<const uint8_t*>(m);
}

// Writes the image next to its final name and renames it into place.
bool store_image(const std::string& dir, ImageHeader h, const uint8_t* image) {
  if (dir.empty() || !make_dirs(dir)) return false;
  h.image_hash = content_hash(image, h.image_bytes);
  const std::string path = image_path(dir, h);
  const std::string tmp = path + ".tmp" + std::to_string(static_cast<long long>(getpid()));
  FILE* f = fopen(tmp.c_str(), "wb");
  if (f == nullptr) return false;
  const bool ok = fwrite(&h, sizeof(h), 1, f) == 1 && fwrite(image, 1, h.image_bytes, f) == h.image_bytes;
  if (fclose(f) != 0 || !ok || rename(tmp.c_str(), path.c_str()) != 0) {
    unlink(tmp.c_str());
    return false;
  }
  return true;
}

bool init_context(native_gpu* g, int device) {
  g->device = device;
  if (!cuda_ok(g, cudaSetDevice(device), "cudaSetDevice")) return false;
  cudaDeviceProp prop;
  if (!cuda_ok(g, cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties")) return false;
  if (prop.major != 10 || prop.minor != 0) {
    fprintf(stderr, "vocalarc-b200: device %d is sm_%d%d; these kernels need sm_100a\n", device, prop.major,
            prop.minor);
    return false;
  }
  snprintf(g->device_name, sizeof(g->device_name), "%s", prop.name);
  g->sm_count = prop.multiProcessorCount;
  g->debug = getenv("VOCALARC_GPU_DEBUG") != nullptr;
  const char* fail = getenv("VOCALARC_B200_FAIL_AT");
  g->fail_at = fail != nullptr ? atoll(fail) : 0;
  const char* prec = getenv("VOCALARC_B200_PRECISION");
  g->bf16 = prec != nullptr && strcmp(prec, "bf16") == 0;
  if (!cuda_ok(g, cudaStreamCreateWithFlags(&g->stream, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
  if (!cuda_ok(g, cudaMalloc(reinterpret_cast<void**>(&g->d_err), sizeof(int)), "cudaMalloc(err)") ||
      !cuda_ok(g, cudaMemset(g->d_err, 0, sizeof(int)), "cudaMemset(err)"))
    return false;
  // Periodic Hann window exactly as stft_channels computes it (vocalarc_separation.c:1052).
  std::vector<float> window(kNfft);
  for (int i = 0; i < kNfft; ++i)
    window[i] = 0.5f - 0.5f * cosf(static_cast<float>(2.0 * 3.141592653589793238462643383279502884 * i / kNfft));
  std::vector<float2> tw(1025);
  for (int k = 0; k <= 1024; ++k) {
    const double a = 2.0 * 3.141592653589793238462643383279502884 * k / 2048.0;
    tw[k] = make_float2(static_cast<float>(cos(a)), static_cast<float>(-sin(a)));
  }
  if (!cuda_ok(g, cudaMalloc(reinterpret_cast<void**>(&g->d_window), kNfft * 4), "cudaMalloc(window)") ||
      !cuda_ok(g, cudaMalloc(reinterpret_cast<void**>(&g->d_twiddle), 1025 * sizeof(float2)), "cudaMalloc(tw)") ||
      !cuda_ok(g, cudaMemcpy(g->d_window, window.data(), kNfft * 4, cudaMemcpyHostToDevice), "window") ||
      !cuda_ok(g, cudaMemcpy(g->d_twiddle, tw.data(), 1025 * sizeof(float2), cudaMemcpyHostToDevice), "twiddle"))
    return false;
  int first[kBands], dims[kBands];
  for (int b = 0; b < kBands; ++b) {
    first[b] = band_first(b);
    dims[b] = 4 * kBandFreqs[b];
  }
  if (!cuda_ok(g, upload_band_tables(first, dims), "band tables")) return false;
  g->enabled = 1;
  return true;
}

void free_model(native_gpu* g) {
  if (g->model_mem != nullptr) cudaFree(g->model_mem);
  g->model_mem = nullptr;
  g->model_loaded = 0;
}

native_gpu* create_on(int device) {
  const char* mode = getenv("VOCALARC_GPU");
  if (mode != nullptr && (strcmp(mode, "off") == 0 || strcmp(mode, "cpu") == 0)) return nullptr;
  native_gpu* g = new native_gpu();
  if (!init_context(g, device)) {
    native_gpu_destroy(g);
    return nullptr;
  }
  return g;
}

const BlockW* cached_block(native_gpu* g, const native_gpu_transformer_weights* w) {
  const uint64_t print = fingerprint(w->qkv, static_cast<size_t>(kQkvDim) * kDim) ^
                         (fingerprint(w->ff2_weight, static_cast<size_t>(kFfDim) * kDim) * 31);
  for (auto& e : g->block_cache)
    if (memcmp(&e.key, w, sizeof(*w)) == 0 && e.print == print && e.bf16 == g->bf16) return &e.w;
  CachedBlock e;
  e.key = *w;
  e.print = print;
  e.bf16 = g->bf16;
  if (!cuda_ok(g, cudaMalloc(&e.mem, kBlockBytes), "cudaMalloc(block weights)")) return nullptr;
  Arena arena{static_cast<char*>(e.mem), kBlockBytes, 0};
  if (!upload_block(g, arena, *w, e.w)) {
    cudaFree(e.mem);
    return nullptr;
  }
  g->block_cache.push_back(e);
  return &g->block_cache.back().w;
}

bool active(const native_gpu* g) { return g != nullptr && g->enabled; }

}  // namespace

namespace vab {
// Read-only view of a provider for entry points defined in other translation
// units: its device, stream and the window / twiddle tables made at creation.
bool provider_view(native_gpu* g, int* device, cudaStream_t* stream, const float** window, const float2** twiddle) {
  if (!active(g)) return false;
  *device = g->device;
  *stream = g->stream;
  *window = g->d_window;
  *twiddle = g->d_twiddle;
  return true;
}

// A launch made by an entry point of another translation unit on this
// provider's stream goes through the same bookkeeping as the provider's own:
// an error disables the provider, the launch is counted and traced.
bool provider_launched(native_gpu* g, cudaError_t e, const char* what) { return launched(g, e, what); }
}  // namespace vab

// ==================================================================== C ABI
extern "C" {

native_gpu* native_gpu_create(void) {
  int device = 0;
  const char* d = getenv("VOCALARC_GPU_DEVICE");
  if (d != nullptr && d[0] != '\0') device = atoi(d);
  return create_on(device);
}

native_gpu* vocalarc_b200_create(int device) { return create_on(device); }

void native_gpu_destroy(native_gpu* g) {
  if (g == nullptr) return;
  cudaSetDevice(g->device);
  if (g->stream != nullptr) cudaStreamSynchronize(g->stream);
  if (g->seam_peer != nullptr) cudaIpcCloseMemHandle(g->seam_peer);
  void* ptrs[] = {g->x, g->x_alt, g->x16, g->row_inv, g->qkv, g->attn, g->gates, g->spec, g->mask, g->frames_buf,
                  g->seg_out, g->audio_in, g->audio_out, g->d_tiles1, g->d_tiles2, g->d_err, g->d_window,
                  g->d_twiddle, g->d_rope, g->abi_mask_mem, g->seam_out, g->seam_in, g->tta_in, g->tta_out,
                  g->x16_alt, g->row_inv_alt};
  for (void* p : ptrs)
    if (p != nullptr) cudaFree(p);
  for (auto& e : g->block_cache) cudaFree(e.mem);
  free_model(g);
  for (cudaEvent_t ev : g->event_pool) cudaEventDestroy(ev);
  if (g->trace_base != nullptr) cudaEventDestroy(g->trace_base);
  if (g->stream != nullptr) cudaStreamDestroy(g->stream);
  delete g;
}

int native_gpu_matmul(native_gpu* gpu, int64_t rows, int in, int out, const float* input, const float* packed_weight,
                      const float* bias, float* output) {
  (void)gpu; (void)rows; (void)in; (void)out; (void)input; (void)packed_weight; (void)bias; (void)output;
  return 0;
}

const char* native_gpu_backend(const native_gpu* gpu) { return active(gpu) ? "native-cuda-sm100a" : "native-cpu"; }

const char* native_gpu_device(const native_gpu* gpu) { return active(gpu) ? gpu->device_name : "none"; }

int native_gpu_uses_full_batches(const native_gpu* gpu) { return active(gpu) ? 1 : 0; }

int native_gpu_can_use_full_batches(const native_gpu* gpu, int frames) {
  if (!active(gpu) || frames <= 0) return 0;
  if (env_is_off("VOCALARC_GPU_FULL_BATCHES")) return 0;
  cudaSetDevice(gpu->device);
  size_t free_b = 0, total_b = 0;
  if (cudaMemGetInfo(&free_b, &total_b) != cudaSuccess || free_b == 0) return 0;
  const double tokens = static_cast<double>(kBands) * frames;
  double need = tokens * (kDim * 4.0 * 2 + kDim * 2 + kQkvDim * 2 + kDimInner * 2 + kHeads * 4);
  need -= gpu->ws_tokens * (kDim * 4.0 * 2 + kDim * 2 + kQkvDim * 2 + kDimInner * 2 + kHeads * 4);
  need += frames * (kFreqBins * 16.0 * 2);                 // mask buffers
  need += 32.0 * kBlockBytes + mask_bytes_estimate();      // converted weights
  need += 512.0 * 1024 * 1024;
  return need < static_cast<double>(free_b) * 0.9 ? 1 : 0;
}

int native_gpu_transformer(native_gpu* g, int sequences, int length, float* data, float* normed, float* qkv,
                           float* attention_output, float* gates, const native_gpu_transformer_weights* weights) {
  (void)normed; (void)qkv; (void)attention_output; (void)gates;
  if (!active(g) || sequences <= 0 || length <= 0 || weights == nullptr || g->resident_active) return 0;
  if (!abi_step(g, "transformer")) return 0;
  cudaSetDevice(g->device);
  const long long tokens = static_cast<long long>(sequences) * length;
  if (!ensure_tokens(g, tokens)) return 0;
  const BlockW* w = cached_block(g, weights);
  if (w == nullptr) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(g->x, data, tokens * kDim * 4, cudaMemcpyHostToDevice, g->stream), "H2D data"))
    return 0;
  g->stats_valid = 0;
  AxisPlan ax{1, length, sequences, 1, sequences, length, 1, length};
  if (!run_block(g, *w, tokens, ax)) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(data, g->x, tokens * kDim * 4, cudaMemcpyDeviceToHost, g->stream), "D2H data"))
    return 0;
  return sync_and_check(g, "transformer") ? 1 : 0;
}

int native_gpu_resident_begin(native_gpu* g, int sequences, int length, const float* data) {
  if (!active(g) || sequences <= 0 || length <= 0 || g->resident_active || data == nullptr) return 0;
  if (!abi_step(g, "resident begin")) return 0;
  cudaSetDevice(g->device);
  const long long tokens = static_cast<long long>(sequences) * length;
  if (!ensure_tokens(g, tokens)) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(g->x, data, tokens * kDim * 4, cudaMemcpyHostToDevice, g->stream), "H2D begin"))
    return 0;
  g->stats_valid = 0;
  if (!sync_and_check(g, "resident begin")) return 0;
  g->resident_active = 1;
  g->resident_tokens = tokens;
  g->phys_s = sequences;
  g->phys_l = length;
  g->transposed = 0;
  return 1;
}

int native_gpu_resident_transformer(native_gpu* g, int sequences, int length,
                                    const native_gpu_transformer_weights* weights) {
  if (!active(g) || !g->resident_active || weights == nullptr ||
      static_cast<long long>(sequences) * length != g->resident_tokens)
    return 0;
  if (!abi_step(g, "resident transformer")) return 0;
  cudaSetDevice(g->device);
  AxisPlan ax;
  if (!g->transposed && sequences == g->phys_s && length == g->phys_l) {
    ax = AxisPlan{1, g->phys_l, g->phys_s, 1, sequences, length, 1, g->phys_l};
  } else if (g->transposed && sequences == g->phys_l && length == g->phys_s) {
    ax = AxisPlan{2, g->phys_l, g->phys_s, 1, sequences, length, g->phys_l, g->phys_s};
  } else {
    return 0;
  }
  const BlockW* w = cached_block(g, weights);
  if (w == nullptr) return 0;
  return run_block(g, *w, g->resident_tokens, ax) ? 1 : 0;
}

int native_gpu_resident_transpose(native_gpu* g, int sequences, int length) {
  if (!active(g) || !g->resident_active || static_cast<long long>(sequences) * length != g->resident_tokens) return 0;
  if (!abi_step(g, "resident transpose")) return 0;
  const int ls = g->transposed ? g->phys_l : g->phys_s;
  const int ll = g->transposed ? g->phys_s : g->phys_l;
  if (sequences != ls || length != ll) return 0;
  g->transposed ^= 1;
  return 1;
}

int native_gpu_resident_end(native_gpu* g, float* data) {
  if (!active(g) || !g->resident_active) return 0;
  if (!abi_step(g, "resident end")) return 0;
  cudaSetDevice(g->device);
  g->resident_active = 0;
  const float* src = g->x;
  if (g->transposed) {
    if (!launched(g, launch_transpose_tokens(g->x, g->x_alt, g->phys_s, g->phys_l, g->stream), "transpose")) return 0;
    src = g->x_alt;
  }
  if (!cuda_ok(g, cudaMemcpyAsync(data, src, g->resident_tokens * kDim * 4, cudaMemcpyDeviceToHost, g->stream),
               "D2H end"))
    return 0;
  return sync_and_check(g, "resident end") ? 1 : 0;
}

int native_gpu_resident_mask(native_gpu* g, int frames, const float* final_gamma, float* mask,
                             const native_gpu_mask_band* bands, int band_count) {
  if (!active(g) || !g->resident_active || frames <= 0 || bands == nullptr || band_count != kBands ||
      final_gamma == nullptr || mask == nullptr)
    return 0;
  if (g->resident_tokens != static_cast<long long>(frames) * kBands) return 0;
  if (!abi_step(g, "resident mask")) return 0;
  bool frame_major;
  if (g->phys_s == kBands && g->phys_l == frames)
    frame_major = false;
  else if (g->phys_s == frames && g->phys_l == kBands)
    frame_major = true;
  else
    return 0;
  for (int b = 0; b < kBands; ++b)
    if (bands[b].input_dim != 4 * kBandFreqs[b] || bands[b].first_frequency != band_first(b)) return 0;
  cudaSetDevice(g->device);
  const uint64_t print = fingerprint(bands[0].first_weight, static_cast<size_t>(kFfDim) * kDim) ^
                         fingerprint(bands[89].second_weight, static_cast<size_t>(2 * 516) * kFfDim) ^
                         fingerprint(final_gamma, kDim);
  if (g->abi_mask_mem == nullptr || g->abi_mask_print != print || g->abi_mask_bf16 != g->bf16) {
    if (g->abi_mask_mem != nullptr) cudaFree(g->abi_mask_mem);
    g->abi_mask_mem = nullptr;
    const size_t bytes = mask_bytes_estimate();
    if (!cuda_ok(g, cudaMalloc(&g->abi_mask_mem, bytes), "cudaMalloc(mask weights)")) return 0;
    Arena arena{static_cast<char*>(g->abi_mask_mem), bytes, 0};
    if (!upload_mask(g, arena, bands, final_gamma, g->abi_mask)) return 0;
    g->abi_mask_print = print;
    g->abi_mask_bf16 = g->bf16;
    g->tiles_frames = 0;
  }
  if (!ensure_frames(g, frames)) return 0;
  if (!run_mask(g, g->abi_mask, 1, frames, frame_major, true, g->mask)) return 0;
  const size_t bytes = static_cast<size_t>(frames) * kFreqBins * 4 * 4;
  if (!cuda_ok(g, cudaMemcpyAsync(mask, g->mask, bytes, cudaMemcpyDeviceToHost, g->stream), "D2H mask")) return 0;
  if (!sync_and_check(g, "resident mask")) return 0;
  g->resident_active = 0;
  return 1;
}

// ------------------------------------------------------------------ extension
int vocalarc_b200_load_model(native_gpu* g, const void* pack, size_t bytes) {
  if (!active(g) || pack == nullptr || bytes < 64) return 0;
  cudaSetDevice(g->device);
  PackView v;
  if (!parse_pack_view(pack, bytes, v)) return 0;
  free_model(g);
  if (!cuda_ok(g, cudaMalloc(&g->model_mem, kModelBytes), "cudaMalloc(model)")) return 0;
  char* base = static_cast<char*>(g->model_mem);
  // Layout pass: every device pointer and tensor map; no weight is touched.
  uint64_t h[kModelTasks];
  for (int t = 0; t < kModelTasks; ++t)
    if (!model_task(g, v, t, base, nullptr, true, true, g->blocks, g->band, g->maskw, &h[t])) return 0;
  const uint64_t layout = fold_layout(h);
  const ImageHeader want = image_header(content_hash(pack, bytes), bytes, layout, g->bf16);
  const std::string dir = image_cache_dir();
  g->model_from_cache = 0;
  size_t mapped = 0;
  const uint8_t* cached = dir.empty() ? nullptr : map_image(image_path(dir, want), want, &mapped);
  if (cached != nullptr) {
    const bool ok = cuda_ok(g, cudaMemcpy(g->model_mem, cached + sizeof(ImageHeader), kModelBytes,
                                          cudaMemcpyHostToDevice), "upload model image");
    munmap(const_cast<uint8_t*>(cached), mapped);
    if (!ok) return 0;
    g->model_from_cache = 1;
  } else {
    std::vector<uint8_t> image(kModelBytes, 0);
    uint64_t built = 0;
    if (!build_image(g, v, base, image.data(), load_threads(), &built) || built != layout) {
      fprintf(stderr, "vocalarc-b200: model conversion failed\n");
      return 0;
    }
    if (!cuda_ok(g, cudaMemcpy(g->model_mem, image.data(), kModelBytes, cudaMemcpyHostToDevice), "upload model image"))
      return 0;
    if (!dir.empty() && !store_image(dir, want, image.data()))
      fprintf(stderr, "vocalarc-b200: could not write the converted model to %s\n", dir.c_str());
  }
  g->tiles_frames = 0;
  g->model_hash = want.pack_hash;
  g->model_loaded = 1;
  return 1;
}

int vocalarc_b200_load_model_file(native_gpu* g, const char* path) {
  if (!active(g) || path == nullptr) return 0;
  const int fd = open(path, O_RDONLY);
  if (fd < 0) {
    fprintf(stderr, "vocalarc-b200: cannot open %s\n", path);
    return 0;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 64) {
    close(fd);
    return 0;
  }
  void* m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (m == MAP_FAILED) return 0;
  const int ok = vocalarc_b200_load_model(g, m, static_cast<size_t>(st.st_size));
  munmap(m, static_cast<size_t>(st.st_size));
  return ok;
}

int vocalarc_b200_model_from_cache(const native_gpu* g) { return g != nullptr && g->model_loaded ? g->model_from_cache : 0; }

int vocalarc_b200_model_image(const void* pack, size_t bytes, int bf16, int threads, void* out, size_t capacity,
                              size_t* image_bytes) {
  if (image_bytes != nullptr) *image_bytes = kModelBytes;
  if (out == nullptr) return 1;
  if (capacity < kModelBytes) return 0;
  PackView v;
  if (!parse_pack_view(pack, bytes, v)) return 0;
  native_gpu host_only;   // conversion settings only; no CUDA call is made
  host_only.bf16 = bf16 ? 1 : 0;
  host_only.enabled = 1;
  memset(out, 0, kModelBytes);
  uint64_t layout = 0;
  return build_image(&host_only, v, kHostOnlyBase, static_cast<uint8_t*>(out), threads > 0 ? threads : load_threads(),
                     &layout)
             ? 1
             : 0;
}

int vocalarc_b200_store_model_image(const void* pack, size_t bytes, int bf16, char* path_out, int capacity) {
  const std::string dir = image_cache_dir();
  PackView v;
  if (dir.empty() || !parse_pack_view(pack, bytes, v)) return 0;
  native_gpu host_only;
  host_only.bf16 = bf16 ? 1 : 0;
  host_only.enabled = 1;
  std::vector<uint8_t> image(kModelBytes, 0);
  uint64_t layout = 0;
  if (!build_image(&host_only, v, kHostOnlyBase, image.data(), load_threads(), &layout)) return 0;
  const ImageHeader h = image_header(content_hash(pack, bytes), bytes, layout, host_only.bf16);
  if (!store_image(dir, h, image.data())) return 0;
  if (path_out != nullptr && capacity > 0) snprintf(path_out, static_cast<size_t>(capacity), "%s", image_path(dir, h).c_str());
  return 1;
}

int vocalarc_b200_set_precision(native_gpu* g, int bf16) {
  if (!active(g)) return 0;
  g->bf16 = bf16 ? 1 : 0;
  g->block_cache.clear();
  return 1;
}

int vocalarc_b200_separate_device(native_gpu* g, const float* d_audio, int tracks, int length, int chunked,
                                  int chunk_samples, int model_batch, float* d_vocals) {
  if (!active(g) || !abi_step(g, "separate")) return 0;
  cudaSetDevice(g->device);
  return separate_device_impl(g, d_audio, tracks, length, chunked, chunk_samples, model_batch, d_vocals) ? 1 : 0;
}

static int separate_host(native_gpu* g, const float* audio, int length, int chunked, int chunk_samples,
                         int model_batch, float* vocals) {
  if (!active(g) || audio == nullptr || vocals == nullptr || length <= 0) return 0;
  if (!abi_step(g, "separate")) return 0;
  cudaSetDevice(g->device);
  const long long n = 2ll * length;
  if (!ensure_audio(g, n)) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(g->audio_in, audio, n * 4, cudaMemcpyHostToDevice, g->stream), "H2D audio")) return 0;
  if (!separate_device_impl(g, g->audio_in, 1, length, chunked, chunk_samples, model_batch, g->audio_out)) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(vocals, g->audio_out, n * 4, cudaMemcpyDeviceToHost, g->stream), "D2H vocals"))
    return 0;
  return sync_and_check(g, "separate") ? 1 : 0;
}

int vocalarc_b200_separate(native_gpu* g, const float* audio, int length, float* vocals) {
  return separate_host(g, audio, length, 0, 0, 1, vocals);
}

int vocalarc_b200_separate_chunked(native_gpu* g, const float* audio, int length, int chunk_samples, int model_batch,
                                   float* vocals) {
  return separate_host(g, audio, length, 1, chunk_samples, model_batch, vocals);
}

// ------------------------------------------------------------------ sequence parallelism
int vocalarc_b200_sp_plan(int count, int frames, int phase, long long* out, int capacity) {
  if (count < 1 || count > kBands || frames < count || phase < 0 || phase > 3) return -1;
  const std::vector<SpCopy> plan = sp_plan(count, frames, phase);
  if (out != nullptr) {
    if (capacity < static_cast<int>(plan.size())) return -1;
    for (size_t i = 0; i < plan.size(); ++i) {
      const SpCopy& c = plan[i];
      const long long v[8] = {c.src, c.dst, c.src_row, c.src_pitch, c.dst_row, c.dst_pitch, c.width, c.height};
      memcpy(out + 8 * i, v, sizeof(v));
    }
  }
  return static_cast<int>(plan.size());
}

int vocalarc_b200_separate_sp(native_gpu* const* gpus, int count, const float* audio, int length, float* vocals) {
  if (gpus == nullptr || count < 1 || count > kBands || audio == nullptr || vocals == nullptr || length <= 0) return 0;
  const int frames = length / kHop + 1;
  if (frames < count) {
    fprintf(stderr, "vocalarc-b200: %d frames cannot be split over %d providers\n", frames, count);
    return 0;
  }
  for (int r = 0; r < count; ++r) {
    if (!active(gpus[r]) || !gpus[r]->model_loaded || gpus[r]->bf16 != gpus[0]->bf16 || gpus[r]->resident_active ||
        gpus[r]->model_hash != gpus[0]->model_hash) {
      fprintf(stderr, "vocalarc-b200: provider %d of the split is not ready (model, precision or open session)\n", r);
      return 0;
    }
    for (int q = 0; q < r; ++q)
      if (gpus[q] == gpus[r]) return 0;
  }
  native_gpu* g0 = gpus[0];
  const long long full = static_cast<long long>(kBands) * frames;
  // Every allocation happens before any work is queued.
  for (int r = 0; r < count; ++r) {
    native_gpu* g = gpus[r];
    cudaSetDevice(g->device);
    if (!ensure_sp(g, full) || !ensure_rope(g, frames > kBands ? frames : kBands)) return 0;
    for (int q = 0; q < count; ++q) {
      if (gpus[q]->device == g->device) continue;
      int can = 0;
      // Direct peer reads where the pair supports them.  An error left by
      // earlier work is reported, not swallowed: only the error of the enable
      // call itself is cleared below.
      const cudaError_t pending = cudaPeekAtLastError();
      if (pending != cudaSuccess) {
        cuda_ok(g, pending, "earlier CUDA call (before enabling peer access)");
        return 0;
      }
      if (cudaDeviceCanAccessPeer(&can, g->device, gpus[q]->device) != cudaSuccess || !can) {
        (void)cudaGetLastError();
        continue;   // the copies between this pair are staged by the driver
      }
      const cudaError_t e = cudaDeviceEnablePeerAccess(gpus[q]->device, 0);
      if (e != cudaSuccess) {
        (void)cudaGetLastError();   // exactly the error of the enable call
        if (e != cudaErrorPeerAccessAlreadyEnabled)
          fprintf(stderr, "vocalarc-b200: peer access %d -> %d refused (%s); copies are staged by the driver\n",
                  g->device, gpus[q]->device, cudaGetErrorString(e));
      }
    }
  }
  cudaSetDevice(g0->device);
  if (!ensure_frames(g0, frames) || !ensure_audio(g0, 2ll * length) || !ensure_mask_tiles(g0, frames, g0->maskw))
    return 0;
  std::vector<cudaEvent_t> ev(count, nullptr);
  bool ok = true;
  for (int r = 0; r < count && ok; ++r) {
    cudaSetDevice(gpus[r]->device);
    ok = cuda_ok(gpus[r], cudaEventCreateWithFlags(&ev[r], cudaEventDisableTiming), "cudaEventCreate");
  }
  auto record = [&](int r) {
    cudaSetDevice(gpus[r]->device);
    return cuda_ok(gpus[r], cudaEventRecord(ev[r], gpus[r]->stream), "cudaEventRecord");
  };
  // Front end on rank 0: STFT, band split and row statistics of the whole clip.
  if (ok) {
    cudaSetDevice(g0->device);
    ok = cuda_ok(g0, cudaMemcpyAsync(g0->audio_in, audio, 2ll * length * 4, cudaMemcpyHostToDevice, g0->stream),
                 "H2D audio") &&
         launched(g0, launch_stft(g0->audio_in, whole_clip_map(length), 1, frames, g0->d_window, g0->d_twiddle,
                                  g0->spec, g0->stream),
                  "stft") &&
         launched(g0, launch_band_split(g0->spec, 1, frames, g0->band.wt, g0->band.wt_off, g0->band.gamma,
                                        g0->band.gamma_off, g0->band.bias, g0->x, g0->stream),
                  "band split");
    g0->stats_valid = 0;
    ok = ok && ensure_stats(g0, full) && record(0) && sp_exchange(gpus, count, frames, 0, ev);
  }
  for (int layer = 0; layer < kDepth && ok; ++layer) {
    for (int r = 0; r < count && ok; ++r) {   // time axis on band ranges
      native_gpu* g = gpus[r];
      const int nb = sp_band_lo(r + 1, count) - sp_band_lo(r, count);
      cudaSetDevice(g->device);
      ok = run_block(g, g->blocks[layer][0], static_cast<long long>(nb) * frames,
                     AxisPlan{1, frames, nb, 1, nb, frames, 1, frames}) &&
           record(r);
    }
    ok = ok && sp_exchange(gpus, count, frames, 1, ev);
    for (int r = 0; r < count && ok; ++r) {   // band axis on frame ranges
      native_gpu* g = gpus[r];
      const int nf = sp_frame_lo(r + 1, count, frames) - sp_frame_lo(r, count, frames);
      cudaSetDevice(g->device);
      ok = run_block(g, g->blocks[layer][1], static_cast<long long>(kBands) * nf,
                     AxisPlan{2, nf, kBands, 1, nf, kBands, nf, kBands}) &&
           record(r);
    }
    ok = ok && sp_exchange(gpus, count, frames, layer + 1 < kDepth ? 2 : 3, ev);
  }
  // Mask head and iSTFT on rank 0.
  if (ok) {
    cudaSetDevice(g0->device);
    ok = run_mask(g0, g0->maskw, 1, frames, false, false, g0->mask) &&
         launched(g0, launch_istft_frames(g0->spec, g0->mask, 1, frames, g0->d_window, g0->d_twiddle, g0->frames_buf,
                                          g0->stream),
                  "istft") &&
         launched(g0, launch_overlap_add(g0->frames_buf, 1, frames, length, g0->d_window, g0->audio_out, g0->stream),
                  "overlap-add") &&
         cuda_ok(g0, cudaMemcpyAsync(vocals, g0->audio_out, 2ll * length * 4, cudaMemcpyDeviceToHost, g0->stream),
                 "D2H vocals");
  }
  // Every stream drains (also on failure) before the buffers are put back in order.
  for (int r = 0; r < count; ++r) {
    native_gpu* g = gpus[r];
    cudaSetDevice(g->device);
    if (!sync_and_check(g, "separate_sp")) ok = false;
    if (g->sp_parity) sp_swap(g);
    g->stats_valid = 0;
    if (ev[r] != nullptr) cudaEventDestroy(ev[r]);
  }
  return ok ? 1 : 0;
}

// ------------------------------------------------------------------ chunk ranges
// One track's chunks split into contiguous ranges, one per GPU.  A range owns
// the padded samples [c0 * step, c1 * step) (the last range: to the padded
// end); its last chunk reaches `seam` = chunk - step samples further, and those
// partial overlap-add sums are the only data that crosses to the next range.

int vocalarc_b200_chunk_plan(int length, int chunk_samples, int* chunks, int* step, int* border, int* seam) {
  if (length <= 0) return 0;
  const int chunk = chunk_samples > 0 ? chunk_samples : 881559;
  const int st = chunk / 2;
  const int bd = chunk - st;
  const bool padded = length > 2 * bd && bd > 0;
  const long long plen = padded ? static_cast<long long>(length) + 2 * bd : length;
  if (st <= 0 || plen > 0x7FFFFFFFLL) return 0;
  if (chunks != nullptr) *chunks = static_cast<int>((plen + st - 1) / st);
  if (step != nullptr) *step = st;
  if (border != nullptr) *border = padded ? bd : 0;
  if (seam != nullptr) *seam = chunk - st;
  return 1;
}

int vocalarc_b200_range_forward(native_gpu* g, const float* d_audio, int length, int chunk_samples, int model_batch,
                                int chunk_begin, int chunk_end) {
  if (!active(g) || d_audio == nullptr) return 0;
  if (!g->model_loaded) {
    fprintf(stderr, "vocalarc-b200: no model loaded (vocalarc_b200_load_model)\n");
    return 0;
  }
  int chunks = 0, step = 0, border = 0, seam = 0;
  if (!vocalarc_b200_chunk_plan(length, chunk_samples, &chunks, &step, &border, &seam)) return 0;
  // Ranges hold at least two chunks (unless one range covers the track), so a
  // seam only ever crosses to the next range.
  if (chunk_begin < 0 || chunk_end > chunks || chunk_end - chunk_begin < (chunk_end - chunk_begin == chunks ? 1 : 2)) {
    fprintf(stderr, "vocalarc-b200: chunk range [%d, %d) invalid for %d chunks (ranges need >= 2 chunks)\n",
            chunk_begin, chunk_end, chunks);
    return 0;
  }
  cudaSetDevice(g->device);
  const int chunk = chunk_samples > 0 ? chunk_samples : 881559;
  const int frames = chunk / kHop + 1;
  const int plen = border > 0 ? length + 2 * border : length;
  const int n = chunk_end - chunk_begin;
  g->range_ready = 0;
  g->has_seam_in = 0;
  if (!ensure_seg(g, static_cast<long long>(n) * 2 * chunk)) return 0;
  if (g->seam_cap < 3ll * seam) {
    g->seam_cap = 0;
    if (!grow(g, &g->seam_out, static_cast<size_t>(seam) * 3 * 4, "cudaMalloc(seam_out)") ||
        !grow(g, &g->seam_in, static_cast<size_t>(seam) * 3 * 4, "cudaMalloc(seam_in)"))
      return 0;
    g->seam_cap = 3ll * seam;
  }
  const int per_pass = max_segments(g, frames, chunk);
  for (int c = chunk_begin; c < chunk_end; c += per_pass) {
    const int m = chunk_end - c < per_pass ? chunk_end - c : per_pass;
    const SegmentMap mm = demix_map(length, chunk, border, plen, step, c);
    if (!forward_segments(g, d_audio, mm, m, frames, g->seg_out + static_cast<long long>(c - chunk_begin) * 2 * chunk))
      return 0;
  }
  g->range_length = length;
  g->range_chunk = chunk;
  g->range_step = step;
  g->range_border = border;
  g->range_plen = plen;
  g->range_chunks = chunks;
  g->range_batch = model_batch < 1 ? 1 : model_batch;
  g->range_c0 = chunk_begin;
  g->range_c1 = chunk_end;
  if (chunk_end < chunks) {
    const SegmentMap dm = demix_map(length, chunk, border, plen, step, 0);
    DemixRange r{chunk_begin, chunk_end, chunk_end * step, chunk_end * step + seam, nullptr, 0, 0, g->seam_out, nullptr};
    if (!launched(g, launch_demix_range(g->seg_out, dm, chunks, g->range_batch, r, g->stream), "demix seam")) return 0;
  }
  // The seam is read by another provider or process once this returns.
  if (!sync_and_check(g, "range forward")) return 0;
  g->range_ready = 1;
  return 1;
}

int vocalarc_b200_range_owned(const native_gpu* g, int* s0, int* s1) {
  if (!active(g) || !g->range_ready) return 0;
  const int p0 = g->range_c0 * g->range_step;
  const int p1 = g->range_c1 < g->range_chunks ? g->range_c1 * g->range_step : g->range_plen;
  const int a = p0 - g->range_border, b = p1 - g->range_border;
  if (s0 != nullptr) *s0 = a < 0 ? 0 : (a > g->range_length ? g->range_length : a);
  if (s1 != nullptr) *s1 = b < 0 ? 0 : (b > g->range_length ? g->range_length : b);
  return 1;
}

int vocalarc_b200_range_seam_export(native_gpu* g, void* handle) {
  if (!active(g) || !g->range_ready || handle == nullptr || g->range_c1 >= g->range_chunks) return 0;
  cudaSetDevice(g->device);
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  return cuda_ok(g, cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), g->seam_out),
                 "cudaIpcGetMemHandle(seam)")
             ? 1
             : 0;
}

int vocalarc_b200_range_seam_import(native_gpu* g, const void* handle) {
  if (!active(g) || !g->range_ready || handle == nullptr || g->range_c0 == 0) return 0;
  cudaSetDevice(g->device);
  static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(g->seam_peer_handle), "IPC handle size");
  if (g->seam_peer == nullptr || memcmp(g->seam_peer_handle, handle, sizeof(g->seam_peer_handle)) != 0) {
    // A new exported buffer: drop the old mapping, map this one.
    if (g->seam_peer != nullptr) cudaIpcCloseMemHandle(g->seam_peer);
    g->seam_peer = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* peer = nullptr;
    if (!cuda_ok(g, cudaIpcOpenMemHandle(&peer, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle(seam)"))
      return 0;
    g->seam_peer = peer;
    memcpy(g->seam_peer_handle, handle, sizeof(g->seam_peer_handle));
  }
  const size_t bytes = static_cast<size_t>(g->range_chunk - g->range_step) * 3 * 4;
  // Peer copy over NVLink into this GPU's memory; the previous range's
  // provider keeps the buffer until every range has finished.
  const bool ok =
      cuda_ok(g, cudaMemcpyAsync(g->seam_in, g->seam_peer, bytes, cudaMemcpyDefault, g->stream), "seam copy") &&
      sync_and_check(g, "seam copy");
  if (!ok) return 0;
  g->has_seam_in = 1;
  return 1;
}

int vocalarc_b200_range_seam_from(native_gpu* g, const native_gpu* prev) {
  if (!active(g) || !g->range_ready || !active(prev) || !prev->range_ready || g->range_c0 == 0 ||
      prev->range_c1 != g->range_c0)
    return 0;
  cudaSetDevice(g->device);
  const size_t bytes = static_cast<size_t>(g->range_chunk - g->range_step) * 3 * 4;
  const cudaError_t e = prev->device == g->device
                            ? cudaMemcpyAsync(g->seam_in, prev->seam_out, bytes, cudaMemcpyDeviceToDevice, g->stream)
                            : cudaMemcpyPeerAsync(g->seam_in, g->device, prev->seam_out, prev->device, bytes, g->stream);
  if (!cuda_ok(g, e, "seam copy") || !sync_and_check(g, "seam copy")) return 0;
  g->has_seam_in = 1;
  return 1;
}

int vocalarc_b200_range_finish(native_gpu* g, float* d_vocals) {
  if (!active(g) || !g->range_ready || d_vocals == nullptr) return 0;
  if (g->range_c0 > 0 && !g->has_seam_in) {
    fprintf(stderr, "vocalarc-b200: range [%d, %d) finished without the previous range's seam\n", g->range_c0,
            g->range_c1);
    return 0;
  }
  cudaSetDevice(g->device);
  const int seam = g->range_chunk - g->range_step;
  const SegmentMap dm = demix_map(g->range_length, g->range_chunk, g->range_border, g->range_plen, g->range_step, 0);
  const int p0 = g->range_c0 * g->range_step;
  const int p1 = g->range_c1 < g->range_chunks ? g->range_c1 * g->range_step : g->range_plen;
  DemixRange r{g->range_c0, g->range_c1, p0, p1, g->range_c0 > 0 ? g->seam_in : nullptr, p0, seam, nullptr, d_vocals};
  if (!launched(g, launch_demix_range(g->seg_out, dm, g->range_chunks, g->range_batch, r, g->stream), "demix range"))
    return 0;
  return sync_and_check(g, "range finish") ? 1 : 0;
}

int vocalarc_b200_separate_tta(native_gpu* g, const float* audio, int length, int chunk_samples, int model_batch,
                               int bigshifts, int tta, float* vocals) {
  if (!active(g) || audio == nullptr || vocals == nullptr || length <= 0) return 0;
  if (!abi_step(g, "separate")) return 0;
  cudaSetDevice(g->device);
  const int shifts = bigshifts < 1 ? 1 : bigshifts;
  const int variants = tta ? 3 : 1;
  const long long n2 = 2ll * length;
  const long long total = n2 * shifts * variants;
  if (!ensure_audio(g, n2)) return 0;
  if (total > g->ws_tta) {
    g->ws_tta = 0;
    if (!grow(g, &g->tta_in, static_cast<size_t>(total) * 4, "cudaMalloc(tta_in)") ||
        !grow(g, &g->tta_out, static_cast<size_t>(total) * 4, "cudaMalloc(tta_out)"))
      return 0;
    g->ws_tta = total;
  }
  if (!cuda_ok(g, cudaMemcpyAsync(g->audio_in, audio, n2 * 4, cudaMemcpyHostToDevice, g->stream), "H2D audio")) return 0;
  if (!launched(g, launch_tta_inputs(g->audio_in, length, shifts, variants, g->tta_in, g->stream), "tta inputs"))
    return 0;
  // All shifted / swapped / inverted copies go through the chunked forward as
  // one batch of tracks.
  if (!separate_device_impl(g, g->tta_in, shifts * variants, length, 1, chunk_samples, model_batch, g->tta_out))
    return 0;
  if (!launched(g, launch_tta_combine(g->tta_out, length, shifts, tta ? 1 : 0, g->audio_out, g->stream), "tta combine"))
    return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(vocals, g->audio_out, n2 * 4, cudaMemcpyDeviceToHost, g->stream), "D2H vocals"))
    return 0;
  return sync_and_check(g, "separate_tta") ? 1 : 0;
}

int vocalarc_b200_synchronize(native_gpu* g) {
  if (!active(g)) return 0;
  cudaSetDevice(g->device);
  return sync_and_check(g, "synchronize") ? 1 : 0;
}

void* vocalarc_b200_stream(native_gpu* g) { return g == nullptr ? nullptr : static_cast<void*>(g->stream); }

int vocalarc_b200_stage_wait_check(native_gpu* g, int limit_us) {
  if (limit_us < 1 || limit_us > 100000) return -1;
  if (!active(g)) return 0;
  cudaSetDevice(g->device);
  if (!launched(g, launch_wait_check(g->d_err, static_cast<unsigned long long>(limit_us) * 1000ull, g->stream),
                "wait check"))
    return 0;
  return sync_and_check(g, "wait check") ? 1 : 0;
}

int vocalarc_b200_take_device_error(native_gpu* g) {
  if (g == nullptr || g->d_err == nullptr) return -1;
  cudaSetDevice(g->device);
  cudaStreamSynchronize(g->stream);
  int err = 0;
  cudaMemcpy(&err, g->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaMemset(g->d_err, 0, sizeof(int));
  return err;
}

// ------------------------------------------------------------------ trace
long long vocalarc_b200_launch_count(const native_gpu* g) { return g == nullptr ? 0 : g->launches; }

int vocalarc_b200_trace_begin(native_gpu* g) {
  if (!active(g)) return 0;
  cudaSetDevice(g->device);
  if (g->trace_base == nullptr && cudaEventCreate(&g->trace_base) != cudaSuccess) return 0;
  g->trace_entries.clear();
  cudaEventRecord(g->trace_base, g->stream);
  g->trace = 1;
  return 1;
}

int vocalarc_b200_trace_mark(native_gpu* g, const char* what) {
  if (!active(g) || !g->trace) return 0;
  trace_mark(g, what);
  return 1;
}

int vocalarc_b200_trace_end(native_gpu* g, char* out, int capacity) {
  if (!active(g) || !g->trace || out == nullptr || capacity <= 0) return 0;
  cudaSetDevice(g->device);
  g->trace = 0;
  if (!cuda_ok(g, cudaStreamSynchronize(g->stream), "trace")) return 0;
  std::vector<std::string> names;
  std::vector<double> ms;
  std::vector<long long> counts;
  cudaEvent_t prev = g->trace_base;
  for (auto& entry : g->trace_entries) {
    float t = 0.f;
    cudaEventElapsedTime(&t, prev, entry.second);
    prev = entry.second;
    size_t i = 0;
    while (i < names.size() && names[i] != entry.first) ++i;
    if (i == names.size()) {
      names.emplace_back(entry.first);
      ms.push_back(0.0);
      counts.push_back(0);
    }
    ms[i] += t;
    counts[i] += 1;
  }
  g->trace_entries.clear();
  std::string text;
  char line[256];
  for (size_t i = 0; i < names.size(); ++i) {
    snprintf(line, sizeof(line), "%s\t%lld\t%.6f\n", names[i].c_str(), counts[i], ms[i]);
    text += line;
  }
  snprintf(out, static_cast<size_t>(capacity), "%s", text.c_str());
  return 1;
}

// ------------------------------------------------------------------ stages
int vocalarc_b200_stage_gemm(native_gpu* g, int epilogue, const void* a, const void* b, int m, int n, int k,
                             const float* bias, void* out) {
  if (!active(g) || m <= 0 || n <= 0 || n % 256 != 0 || k <= 0 || k % 64 != 0) return 0;
  if (epilogue != kEpiStore && epilogue != kEpiGelu && epilogue != kEpiStoreF32) return 0;
  cudaSetDevice(g->device);
  GemmMaps maps;
  if (!make_map_rows(g, &maps.a, a, m, k, 128) || !make_map_rows(g, &maps.b, b, n, k, 256)) return 0;
  if (epilogue == kEpiStoreF32)
    maps.c = maps.d = maps.a;
  else if (!make_out16_map(g, &maps.c, out, m, n))
    return 0;
  else
    maps.d = maps.c;
  GemmArgs args = uniform_args(g, m, n, k);
  args.out = out;
  args.ldo = n;
  args.bias = bias;
  return launched(g, launch_gemm(epilogue, g->bf16 != 0, maps, args, g->sm_count, g->stream), "stage gemm") ? 1 : 0;
}

int vocalarc_b200_stage_attention(native_gpu* g, const void* qkv, const float* gates, void* out, int d1, int d2,
                                  int d3, int pos_dim) {
  if (!active(g) || d1 <= 0 || d2 <= 0 || d3 <= 0 || (pos_dim != 1 && pos_dim != 2)) return 0;
  cudaSetDevice(g->device);
  CUtensorMap q4;
  const uint64_t dims[4] = {static_cast<uint64_t>(kQkvDim), static_cast<uint64_t>(d1), static_cast<uint64_t>(d2),
                            static_cast<uint64_t>(d3)};
  const uint64_t rb = kQkvDim * 2ull;
  const uint64_t strides[3] = {rb, rb * d1, rb * d1 * d2};
  const uint32_t box[4] = {64u, pos_dim == 1 ? 128u : 1u, pos_dim == 2 ? 128u : 1u, 1u};
  if (!make_tmap_4d(&q4, qkv, 2, dims, strides, box, g->bf16 != 0)) return 0;
  AttnArgs at;
  at.length = pos_dim == 1 ? d1 : d2;
  at.sequences = pos_dim == 1 ? d2 * d3 : d1 * d3;
  at.q_tiles = (at.length + 127) / 128;
  at.pos_dim = pos_dim;
  at.d1 = d1;
  at.d2 = d2;
  at.gates = gates;
  at.out = out;
  at.err = g->d_err;
  return launched(g, launch_attention(g->bf16 != 0, q4, at, g->sm_count, g->stream), "stage attention") ? 1 : 0;
}

int vocalarc_b200_stage_stft(native_gpu* g, const float* audio, int segments, int length, float* spec) {
  if (!active(g) || segments <= 0 || length <= 0) return 0;
  cudaSetDevice(g->device);
  const SegmentMap map = whole_clip_map(length);
  return launched(g, launch_stft(audio, map, segments, length / kHop + 1, g->d_window, g->d_twiddle, spec, g->stream),
                  "stage stft")
             ? 1
             : 0;
}

int vocalarc_b200_stage_istft(native_gpu* g, const float* spec, const float* mask, int segments, int length,
                              float* audio) {
  if (!active(g) || segments <= 0 || length <= 0) return 0;
  cudaSetDevice(g->device);
  const int frames = length / kHop + 1;
  if (!ensure_frames(g, static_cast<long long>(segments) * frames)) return 0;
  if (!launched(g, launch_istft_frames(spec, mask, segments, frames, g->d_window, g->d_twiddle, g->frames_buf,
                                       g->stream),
                "stage istft"))
    return 0;
  return launched(g, launch_overlap_add(g->frames_buf, segments, frames, length, g->d_window, audio, g->stream),
                  "stage ola")
             ? 1
             : 0;
}

int vocalarc_b200_stage_band_split(native_gpu* g, const float* spec, int segments, int frames, float* x) {
  if (!active(g) || !g->model_loaded || segments <= 0 || frames <= 0) return 0;
  cudaSetDevice(g->device);
  return launched(g, launch_band_split(spec, segments, frames, g->band.wt, g->band.wt_off, g->band.gamma,
                                       g->band.gamma_off, g->band.bias, x, g->stream),
                  "stage band split")
             ? 1
             : 0;
}

int vocalarc_b200_stage_block(native_gpu* g, float* x, int segments, int frames, int layer, int axis) {
  if (!active(g) || !g->model_loaded || segments <= 0 || frames <= 0 || layer < 0 || layer >= kDepth || axis < 0 ||
      axis > 1)
    return 0;
  cudaSetDevice(g->device);
  const long long tokens = static_cast<long long>(segments) * kBands * frames;
  if (!ensure_tokens(g, tokens)) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(g->x, x, tokens * kDim * 4, cudaMemcpyDeviceToDevice, g->stream), "D2D")) return 0;
  g->stats_valid = 0;
  if (!run_block(g, g->blocks[layer][axis], tokens, axis == 0 ? time_axis(segments, frames) : band_axis(segments, frames)))
    return 0;
  return cuda_ok(g, cudaMemcpyAsync(x, g->x, tokens * kDim * 4, cudaMemcpyDeviceToDevice, g->stream), "D2D") ? 1 : 0;
}

int vocalarc_b200_stage_mask(native_gpu* g, const float* x, int segments, int frames, float* mask) {
  if (!active(g) || !g->model_loaded || segments <= 0 || frames <= 0) return 0;
  cudaSetDevice(g->device);
  const long long tokens = static_cast<long long>(segments) * kBands * frames;
  if (!ensure_tokens(g, tokens)) return 0;
  if (!cuda_ok(g, cudaMemcpyAsync(g->x, x, tokens * kDim * 4, cudaMemcpyDeviceToDevice, g->stream), "D2D")) return 0;
  g->stats_valid = 0;
  return run_mask(g, g->maskw, segments, frames, false, false, mask) ? 1 : 0;
}

}  // extern "C"
