// Configurable BS-RoFormer stack (vocalarc_b200_stack.h): the forward of
// runtime.cu with the model sizes as parameters -- residual width 256 or 512,
// any band table, any hop, GELU or GEGLU FFN, any mask hidden width.  It runs
// the same kernels: the tcgen05 GEMM (norm-folded operands, fused epilogues),
// the two attention kernels, and the spectral kernels with the hop and width
// passed in.
//
// Differences from the bundled path, all in the orchestration:
//  * residual rows wider than one 256-column tile: the residual GEMM's tiles
//    add their halves of sum x^2 into a per-row float and a small kernel turns
//    it into the RMSNorm factor sqrt(dim)/|x| (and clears it);
//  * GEGLU: the FFN input projection's rows are interleaved (value i, gate i)
//    at load time so one accumulator tile holds whole pairs, and the GEMM
//    epilogue writes value * gelu(gate);
//  * the mask GEMM's GLU scatter takes the band count and tables from global
//    memory instead of the bundled 90-band constant tables.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "vab_internal.h"
#include "vocalarc_b200_stack.h"

using namespace vab;

namespace {

constexpr int kStackQkvRows = kQkvDim + 16;   // q|k|v, 8 gate rows, 8 zero rows

int round16s(int x) { return (x + 15) & ~15; }

// Validated sizes derived from a configuration.
struct StackShape {
  int dim = 0, depth = 0, ff_inner = 0, ff1_rows = 0, geglu = 0, hidden = 0, bands = 0, hop = 0;
  int bins[VOCALARC_B200_STACK_MAX_BANDS];
  int first[VOCALARC_B200_STACK_MAX_BANDS];
  int split_dim = 0;   // sum of 4 w_b
  size_t block_floats = 0, band_floats = 0, mask_floats = 0, total = 0;
};

bool shape_of(const vocalarc_b200_stack_config* c, StackShape& s) {
  if (c == nullptr) return false;
  if (c->dim != 256 && c->dim != 512) return false;
  if (c->depth < 1 || c->depth > 64 || c->heads != kHeads || c->dim_head != kDimHead || c->n_fft != kNfft) return false;
  if (c->geglu != 0 && c->geglu != 1) return false;
  if (c->ff_inner <= 0 || c->ff_inner % (c->geglu ? 128 : 256) != 0 || c->ff_inner > 16384) return false;
  if (c->mask_hidden <= 0 || c->mask_hidden % 256 != 0 || c->mask_hidden > 16384) return false;
  if (c->bands < 1 || c->bands > VOCALARC_B200_STACK_MAX_BANDS || c->hop < 1 || c->hop > kNfft) return false;
  if (c->bf16 != 0 && c->bf16 != 1) return false;
  s.dim = c->dim;
  s.depth = c->depth;
  s.ff_inner = c->ff_inner;
  s.geglu = c->geglu;
  s.ff1_rows = c->ff_inner * (c->geglu ? 2 : 1);
  s.hidden = c->mask_hidden;
  s.bands = c->bands;
  s.hop = c->hop;
  int first = 0;
  s.split_dim = 0;
  for (int b = 0; b < c->bands; ++b) {
    const int w = c->band_bins[b];
    if (w < 1 || w > 129) return false;   // the band-split kernel stages rows of up to 516 floats
    s.bins[b] = w;
    s.first[b] = first;
    first += w;
    s.split_dim += 4 * w;
  }
  if (first != kFreqBins) return false;
  const size_t d = static_cast<size_t>(s.dim);
  s.block_floats = d + static_cast<size_t>(kQkvDim) * d + kHeads * d + kHeads + d * kDimInner + d +
                   static_cast<size_t>(s.ff1_rows) * d + s.ff1_rows + d * s.ff_inner + d;
  s.band_floats = 0;
  s.mask_floats = 0;
  for (int b = 0; b < s.bands; ++b) {
    const size_t db = 4 * static_cast<size_t>(s.bins[b]);
    s.band_floats += db + d * db + d;
    s.mask_floats += static_cast<size_t>(s.hidden) * d + s.hidden + 2 * db * s.hidden + 2 * db;
  }
  s.total = s.block_floats * 2 * s.depth + s.band_floats + d + s.mask_floats;
  return true;
}

struct StackBlock {
  void* qkv = nullptr;
  void* out = nullptr;
  void* ff1 = nullptr;
  void* ff2 = nullptr;
  float* gate_b = nullptr;
  float* ff1_b = nullptr;
  float* ff2_b = nullptr;
  CUtensorMap m_qkv, m_out, m_ff1, m_ff2;
};


}  // namespace

struct vocalarc_b200_stack {
  int device = 0;
  int ok = 0;
  int bf16 = 0;
  int sm_count = 148;
  StackShape shape;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;
  float* d_window = nullptr;
  float2* d_twiddle = nullptr;
  float4* d_rope = nullptr;
  int rope_len = 0;
  // weights
  void* model_mem = nullptr;
  std::vector<StackBlock> blocks;   // [depth][2]
  float* band_wt = nullptr;
  long long* band_wt_off = nullptr;
  float* band_gamma = nullptr;
  int* band_gamma_off = nullptr;
  float* band_bias = nullptr;
  void* w1 = nullptr;
  float* b1 = nullptr;
  void* w2 = nullptr;
  float* b2 = nullptr;
  CUtensorMap m_w1, m_w2;
  int* d_band_first = nullptr;
  int* d_band_dim = nullptr;
  std::vector<int> w2_off, w2_rows;
  int w2_total = 0;
  // mask tile tables (per frame count)
  int tiles_frames = 0;
  int4* d_tiles1 = nullptr;
  int4* d_tiles2 = nullptr;
  int n_tiles1 = 0, n_tiles2 = 0;
  // workspace
  long long ws_tokens = 0;
  float* x = nullptr;
  void* x16 = nullptr;
  float* row_inv = nullptr;
  float* sumsq = nullptr;
  void* wide = nullptr;    // q|k|v, the FFN hidden and the mask hidden, 16-bit
  long long wide_cols = 0;
  void* attn = nullptr;
  float* gates = nullptr;
  long long ws_frames = 0;
  float* spec = nullptr;
  float* mask = nullptr;
  float* frames_buf = nullptr;
  long long ws_audio = 0;
  float* audio_in = nullptr;
  float* audio_out = nullptr;
  // launch accounting and trace
  long long launches = 0;
  int trace = 0;
  cudaEvent_t trace_base = nullptr;
  std::vector<cudaEvent_t> event_pool;
  std::vector<std::pair<const char*, cudaEvent_t>> trace_entries;
};

namespace {

using Stack = vocalarc_b200_stack;

bool sok(Stack* s, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return true;
  fprintf(stderr, "vocalarc-b200 stack: %s failed: %s\n", what, cudaGetErrorString(e));
  s->ok = 0;
  return false;
}

bool slaunched(Stack* s, cudaError_t e, const char* what) {
  if (!sok(s, e, what)) return false;
  ++s->launches;
  if (s->trace) {
    const size_t used = s->trace_entries.size();
    if (used == s->event_pool.size()) {
      cudaEvent_t ev = nullptr;
      if (cudaEventCreate(&ev) != cudaSuccess) return true;
      s->event_pool.push_back(ev);
    }
    cudaEventRecord(s->event_pool[used], s->stream);
    s->trace_entries.emplace_back(what, s->event_pool[used]);
  }
  return true;
}

template <typename P>
bool sgrow(Stack* s, P** ptr, size_t bytes, const char* what) {
  if (*ptr != nullptr) cudaFree(*ptr);
  *ptr = nullptr;
  return sok(s, cudaMalloc(reinterpret_cast<void**>(ptr), bytes), what);
}

void to16s(const float* w, size_t n, bool bf16, std::vector<uint16_t>& out) {
  out.resize(n);
  for (size_t i = 0; i < n; ++i) {
    if (bf16) {
      const __nv_bfloat16 h = __float2bfloat16_rn(w[i]);
      memcpy(&out[i], &h, 2);
    } else {
      const __half h = __float2half_rn(w[i]);
      memcpy(&out[i], &h, 2);
    }
  }
}

struct SArena {
  char* base = nullptr;
  size_t cap = 0, used = 0;
  void* take(size_t bytes) {
    const size_t off = (used + 1023) & ~size_t(1023);
    if (off + bytes > cap) return nullptr;
    used = off + bytes;
    return base + off;
  }
};

bool map_rows(Stack* s, CUtensorMap* map, const void* base, long long rows, int k, int box_rows) {
  return make_tmap_2d(map, base, 2, static_cast<uint64_t>(k), static_cast<uint64_t>(rows),
                      static_cast<uint64_t>(k) * 2, 64, static_cast<uint32_t>(box_rows), 128, s->bf16 != 0);
}

// 16-bit weight matrix W[rows][k] into the arena, with its B-operand map.
bool upload_w16(Stack* s, SArena& arena, const std::vector<float>& w, int rows, int k, int box_rows, void** dst,
                CUtensorMap* map) {
  std::vector<uint16_t> h;
  to16s(w.data(), w.size(), s->bf16 != 0, h);
  *dst = arena.take(h.size() * 2);
  if (*dst == nullptr) return false;
  if (!sok(s, cudaMemcpy(*dst, h.data(), h.size() * 2, cudaMemcpyHostToDevice), "weights")) return false;
  return map_rows(s, map, *dst, rows, k, box_rows);
}

bool upload_fs(Stack* s, SArena& arena, const float* src, size_t count, float** dst) {
  *dst = static_cast<float*>(arena.take(count * 4));
  return *dst != nullptr && sok(s, cudaMemcpy(*dst, src, count * 4, cudaMemcpyHostToDevice), "weights");
}

// W[out][in] with column i scaled by gamma[i] (an RMSNorm gamma folded into the consuming GEMM).
std::vector<float> folded(const float* w, int out, int in, const float* gamma) {
  std::vector<float> r(w, w + static_cast<size_t>(out) * in);
  if (gamma != nullptr)
    for (int o = 0; o < out; ++o)
      for (int i = 0; i < in; ++i) r[static_cast<size_t>(o) * in + i] *= gamma[i];
  return r;
}

bool load_weights(Stack* s, const float* w) {
  const StackShape& sh = s->shape;
  const int d = sh.dim;
  // Device bytes: generous upper bound (16-bit matrices, fp32 vectors, 1 KB alignment per piece).
  const size_t mats16 = static_cast<size_t>(2 * sh.depth) *
                        (static_cast<size_t>(kStackQkvRows) * d + static_cast<size_t>(d) * kDimInner +
                         static_cast<size_t>(sh.ff1_rows) * d + static_cast<size_t>(d) * sh.ff_inner);
  size_t w2_rows_total = 0;
  for (int b = 0; b < sh.bands; ++b) w2_rows_total += round16s(8 * sh.bins[b]);
  const size_t mask16 = static_cast<size_t>(sh.bands) * sh.hidden * d + w2_rows_total * sh.hidden;
  const size_t vec32 = static_cast<size_t>(2 * sh.depth) * (kHeads + sh.ff1_rows + d) +
                       static_cast<size_t>(sh.split_dim) * d + sh.split_dim + static_cast<size_t>(sh.bands) * d +
                       static_cast<size_t>(sh.bands) * sh.hidden + w2_rows_total + 8 * sh.bands + 16;
  const size_t pieces = static_cast<size_t>(2 * sh.depth) * 8 + 16;
  const size_t bytes = mats16 * 2 + mask16 * 2 + vec32 * 4 + pieces * 1024 + (1 << 20);
  if (!sok(s, cudaMalloc(&s->model_mem, bytes), "cudaMalloc(stack weights)")) return false;
  SArena arena{static_cast<char*>(s->model_mem), bytes, 0};

  const float* p = w;
  s->blocks.resize(static_cast<size_t>(2 * sh.depth));
  for (int l = 0; l < sh.depth; ++l)
    for (int a = 0; a < 2; ++a) {
      StackBlock& blk = s->blocks[static_cast<size_t>(2 * l + a)];
      const float* gamma = p;               p += d;
      const float* qkv = p;                 p += static_cast<size_t>(kQkvDim) * d;
      const float* gate_w = p;              p += kHeads * d;
      const float* gate_b = p;              p += kHeads;
      const float* out_w = p;               p += static_cast<size_t>(d) * kDimInner;
      const float* ff_gamma = p;            p += d;
      const float* ff1 = p;                 p += static_cast<size_t>(sh.ff1_rows) * d;
      const float* ff1_b = p;               p += sh.ff1_rows;
      const float* ff2 = p;                 p += static_cast<size_t>(d) * sh.ff_inner;
      const float* ff2_b = p;               p += d;
      // q|k|v and the gate rows, both consuming the attention norm.
      std::vector<float> q(static_cast<size_t>(kStackQkvRows) * d, 0.f);
      std::vector<float> f = folded(qkv, kQkvDim, d, gamma);
      std::copy(f.begin(), f.end(), q.begin());
      f = folded(gate_w, kHeads, d, gamma);
      std::copy(f.begin(), f.end(), q.begin() + static_cast<size_t>(kQkvDim) * d);
      if (!upload_w16(s, arena, q, kStackQkvRows, d, 256, &blk.qkv, &blk.m_qkv)) return false;
      if (!upload_w16(s, arena, folded(out_w, d, kDimInner, nullptr), d, kDimInner, 256, &blk.out, &blk.m_out))
        return false;
      // FFN input projection; GEGLU rows interleaved (value i, gate i).
      std::vector<float> f1 = folded(ff1, sh.ff1_rows, d, ff_gamma), b1(ff1_b, ff1_b + sh.ff1_rows);
      if (sh.geglu) {
        std::vector<float> inter(f1.size()), ib(b1.size());
        for (int i = 0; i < sh.ff_inner; ++i) {
          memcpy(&inter[static_cast<size_t>(2 * i) * d], &f1[static_cast<size_t>(i) * d], d * 4);
          memcpy(&inter[static_cast<size_t>(2 * i + 1) * d], &f1[static_cast<size_t>(sh.ff_inner + i) * d], d * 4);
          ib[2 * i] = b1[i];
          ib[2 * i + 1] = b1[sh.ff_inner + i];
        }
        f1.swap(inter);
        b1.swap(ib);
      }
      if (!upload_w16(s, arena, f1, sh.ff1_rows, d, 256, &blk.ff1, &blk.m_ff1)) return false;
      if (!upload_w16(s, arena, folded(ff2, d, sh.ff_inner, nullptr), d, sh.ff_inner, 256, &blk.ff2, &blk.m_ff2))
        return false;
      if (!upload_fs(s, arena, gate_b, kHeads, &blk.gate_b) || !upload_fs(s, arena, b1.data(), b1.size(), &blk.ff1_b) ||
          !upload_fs(s, arena, ff2_b, d, &blk.ff2_b))
        return false;
    }
  // Band split: W^T [d_b][dim] per band, gammas in bin order, biases [bands][dim].
  std::vector<float> wt(static_cast<size_t>(sh.split_dim) * d), gam(sh.split_dim), bias(static_cast<size_t>(sh.bands) * d);
  std::vector<long long> wt_off(sh.bands);
  std::vector<int> g_off(sh.bands + 1);
  size_t cur_wt = 0;
  int cur_g = 0;
  for (int b = 0; b < sh.bands; ++b) {
    const int db = 4 * sh.bins[b];
    const float* gamma = p;   p += db;
    const float* weight = p;  p += static_cast<size_t>(d) * db;
    const float* bb = p;      p += d;
    wt_off[b] = static_cast<long long>(cur_wt);
    for (int k = 0; k < db; ++k)
      for (int n = 0; n < d; ++n) wt[cur_wt + static_cast<size_t>(k) * d + n] = weight[static_cast<size_t>(n) * db + k];
    cur_wt += static_cast<size_t>(db) * d;
    g_off[b] = cur_g;
    memcpy(&gam[cur_g], gamma, db * 4);
    cur_g += db;
    memcpy(&bias[static_cast<size_t>(b) * d], bb, d * 4);
  }
  g_off[sh.bands] = cur_g;
  if (!upload_fs(s, arena, wt.data(), wt.size(), &s->band_wt) ||
      !upload_fs(s, arena, gam.data(), gam.size(), &s->band_gamma) ||
      !upload_fs(s, arena, bias.data(), bias.size(), &s->band_bias))
    return false;
  s->band_wt_off = static_cast<long long*>(arena.take(sh.bands * 8));
  s->band_gamma_off = static_cast<int*>(arena.take((sh.bands + 1) * 4));
  s->d_band_first = static_cast<int*>(arena.take(sh.bands * 4));
  s->d_band_dim = static_cast<int*>(arena.take(sh.bands * 4));
  if (s->band_wt_off == nullptr || s->band_gamma_off == nullptr || s->d_band_first == nullptr ||
      s->d_band_dim == nullptr)
    return false;
  std::vector<int> dims(sh.bands);
  for (int b = 0; b < sh.bands; ++b) dims[b] = 4 * sh.bins[b];
  if (!sok(s, cudaMemcpy(s->band_wt_off, wt_off.data(), sh.bands * 8, cudaMemcpyHostToDevice), "band tables") ||
      !sok(s, cudaMemcpy(s->band_gamma_off, g_off.data(), (sh.bands + 1) * 4, cudaMemcpyHostToDevice), "band tables") ||
      !sok(s, cudaMemcpy(s->d_band_first, sh.first, sh.bands * 4, cudaMemcpyHostToDevice), "band tables") ||
      !sok(s, cudaMemcpy(s->d_band_dim, dims.data(), sh.bands * 4, cudaMemcpyHostToDevice), "band tables"))
    return false;
  // Mask head: final gamma folded into layer 1; layer-2 rows interleaved (value i, gate i), padded to 16 per band.
  const float* final_gamma = p;
  p += d;
  std::vector<float> all1(static_cast<size_t>(sh.bands) * sh.hidden * d), ball1(static_cast<size_t>(sh.bands) * sh.hidden);
  s->w2_off.assign(sh.bands, 0);
  s->w2_rows.assign(sh.bands, 0);
  s->w2_total = 0;
  for (int b = 0; b < sh.bands; ++b) {
    s->w2_off[b] = s->w2_total;
    s->w2_rows[b] = round16s(8 * sh.bins[b]);
    s->w2_total += s->w2_rows[b];
  }
  std::vector<float> all2(static_cast<size_t>(s->w2_total) * sh.hidden, 0.f), ball2(s->w2_total, 0.f);
  for (int b = 0; b < sh.bands; ++b) {
    const int db = 4 * sh.bins[b];
    const float* w1 = p;  p += static_cast<size_t>(sh.hidden) * d;
    const float* b1 = p;  p += sh.hidden;
    const float* w2 = p;  p += static_cast<size_t>(2 * db) * sh.hidden;
    const float* b2 = p;  p += 2 * db;
    const std::vector<float> f = folded(w1, sh.hidden, d, final_gamma);
    memcpy(&all1[static_cast<size_t>(b) * sh.hidden * d], f.data(), f.size() * 4);
    memcpy(&ball1[static_cast<size_t>(b) * sh.hidden], b1, sh.hidden * 4);
    const size_t off = s->w2_off[b];
    for (int i = 0; i < db; ++i) {
      memcpy(&all2[(off + 2 * i) * sh.hidden], w2 + static_cast<size_t>(i) * sh.hidden, sh.hidden * 4);
      memcpy(&all2[(off + 2 * i + 1) * sh.hidden], w2 + static_cast<size_t>(db + i) * sh.hidden, sh.hidden * 4);
      ball2[off + 2 * i] = b2[i];
      ball2[off + 2 * i + 1] = b2[db + i];
    }
  }
  if (static_cast<size_t>(p - w) != sh.total) return false;
  if (!upload_w16(s, arena, all1, sh.bands * sh.hidden, d, 256, &s->w1, &s->m_w1) ||
      !upload_fs(s, arena, ball1.data(), ball1.size(), &s->b1) ||
      !upload_w16(s, arena, all2, s->w2_total, sh.hidden, 16, &s->w2, &s->m_w2) ||
      !upload_fs(s, arena, ball2.data(), ball2.size(), &s->b2))
    return false;
  return true;
}

bool init_stack(Stack* s, int device) {
  s->device = device;
  if (!sok(s, cudaSetDevice(device), "cudaSetDevice")) return false;
  cudaDeviceProp prop;
  if (!sok(s, cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties")) return false;
  if (prop.major != 10 || prop.minor != 0) {
    fprintf(stderr, "vocalarc-b200 stack: device %d is sm_%d%d; these kernels need sm_100a\n", device, prop.major,
            prop.minor);
    return false;
  }
  s->sm_count = prop.multiProcessorCount;
  if (!sok(s, cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking), "cudaStreamCreate")) return false;
  if (!sok(s, cudaMalloc(reinterpret_cast<void**>(&s->d_err), sizeof(int)), "cudaMalloc(err)") ||
      !sok(s, cudaMemset(s->d_err, 0, sizeof(int)), "cudaMemset(err)"))
    return false;
  // Periodic Hann window and the 2048-point twiddles, as the bundled provider makes them.
  std::vector<float> window(kNfft);
  for (int i = 0; i < kNfft; ++i)
    window[i] = 0.5f - 0.5f * cosf(static_cast<float>(2.0 * 3.141592653589793238462643383279502884 * i / kNfft));
  std::vector<float2> tw(1025);
  for (int k = 0; k <= 1024; ++k) {
    const double a = 2.0 * 3.141592653589793238462643383279502884 * k / 2048.0;
    tw[k] = make_float2(static_cast<float>(cos(a)), static_cast<float>(-sin(a)));
  }
  return sok(s, cudaMalloc(reinterpret_cast<void**>(&s->d_window), kNfft * 4), "cudaMalloc(window)") &&
         sok(s, cudaMalloc(reinterpret_cast<void**>(&s->d_twiddle), 1025 * sizeof(float2)), "cudaMalloc(tw)") &&
         sok(s, cudaMemcpy(s->d_window, window.data(), kNfft * 4, cudaMemcpyHostToDevice), "window") &&
         sok(s, cudaMemcpy(s->d_twiddle, tw.data(), 1025 * sizeof(float2), cudaMemcpyHostToDevice), "twiddle");
}

// RoPE cos/sin table, the bundled provider's (rope_table: apply_rotary,
// vocalarc_separation.c:726-731; fill_frequencies :1312-1314).
bool ensure_rope_s(Stack* s, int positions) {
  if (positions <= s->rope_len) return true;
  const int n = positions < 128 ? 128 : positions;
  const std::vector<float4> table = rope_table(n);
  s->rope_len = 0;
  if (!sgrow(s, &s->d_rope, table.size() * sizeof(float4), "cudaMalloc(rope)")) return false;
  if (!sok(s, cudaMemcpy(s->d_rope, table.data(), table.size() * sizeof(float4), cudaMemcpyHostToDevice), "rope"))
    return false;
  s->rope_len = n;
  return true;
}

bool ensure_tokens_s(Stack* s, long long tokens) {
  const StackShape& sh = s->shape;
  long long wide = kQkvDim;
  if (sh.ff_inner > wide) wide = sh.ff_inner;
  if (sh.hidden > wide) wide = sh.hidden;
  if (tokens <= s->ws_tokens && wide <= s->wide_cols) return true;
  s->ws_tokens = 0;
  const size_t t = static_cast<size_t>(tokens), d = static_cast<size_t>(sh.dim);
  if (!sgrow(s, &s->x, t * d * 4, "cudaMalloc(x)") || !sgrow(s, &s->x16, t * d * 2, "cudaMalloc(x16)") ||
      !sgrow(s, &s->row_inv, t * 4, "cudaMalloc(row_inv)") || !sgrow(s, &s->sumsq, t * 4, "cudaMalloc(sumsq)") ||
      !sgrow(s, &s->wide, t * static_cast<size_t>(wide) * 2, "cudaMalloc(wide)") ||
      !sgrow(s, &s->attn, t * kDimInner * 2, "cudaMalloc(attn)") ||
      !sgrow(s, &s->gates, t * kHeads * 4, "cudaMalloc(gates)"))
    return false;
  if (!sok(s, cudaMemsetAsync(s->sumsq, 0, t * 4, s->stream), "memset(sumsq)")) return false;
  s->ws_tokens = tokens;
  s->wide_cols = wide;
  return true;
}

bool ensure_frames_s(Stack* s, long long seg_frames) {
  if (seg_frames <= s->ws_frames) return true;
  s->ws_frames = 0;
  const size_t f = static_cast<size_t>(seg_frames);
  if (!sgrow(s, &s->spec, f * kFreqBins * 16, "cudaMalloc(spec)") ||
      !sgrow(s, &s->mask, f * kFreqBins * 16, "cudaMalloc(mask)") ||
      !sgrow(s, &s->frames_buf, f * 2 * kNfft * 4, "cudaMalloc(frames)"))
    return false;
  s->ws_frames = seg_frames;
  return true;
}

bool ensure_mask_tiles_s(Stack* s, int frames) {
  if (s->tiles_frames == frames && s->d_tiles1 != nullptr) return true;
  const StackShape& sh = s->shape;
  std::vector<int4> t1, t2;
  for (int b = 0; b < sh.bands; ++b)
    for (int m0 = 0; m0 < frames; m0 += 128) {
      const int mv = frames - m0 < 128 ? frames - m0 : 128;
      for (int n0 = 0; n0 < sh.hidden; n0 += 256) t1.push_back(make_tile(b * frames + m0, b * sh.hidden + n0, n0, mv, 256, b));
      for (int n0 = 0; n0 < s->w2_rows[b]; n0 += 256) {
        const int ns = s->w2_rows[b] - n0 < 256 ? s->w2_rows[b] - n0 : 256;
        t2.push_back(make_tile(b * frames + m0, s->w2_off[b] + n0, n0, mv, ns, b));
      }
    }
  s->tiles_frames = 0;
  if (!sgrow(s, &s->d_tiles1, t1.size() * sizeof(int4), "cudaMalloc(tiles)") ||
      !sgrow(s, &s->d_tiles2, t2.size() * sizeof(int4), "cudaMalloc(tiles)"))
    return false;
  if (!sok(s, cudaMemcpy(s->d_tiles1, t1.data(), t1.size() * sizeof(int4), cudaMemcpyHostToDevice), "tiles") ||
      !sok(s, cudaMemcpy(s->d_tiles2, t2.data(), t2.size() * sizeof(int4), cudaMemcpyHostToDevice), "tiles"))
    return false;
  s->n_tiles1 = static_cast<int>(t1.size());
  s->n_tiles2 = static_cast<int>(t2.size());
  s->tiles_frames = frames;
  return true;
}

bool stack_hook(void* owner, cudaError_t e, const char* what) {
  return slaunched(static_cast<Stack*>(owner), e, what);
}

// One axial block on s->x through the shared orchestration of block.cu
// (x16 / row_inv describe the current x and are left describing the updated x).
bool run_block_s(Stack* s, const StackBlock& w, long long tokens, const AxisPlan& ax) {
  const StackShape& sh = s->shape;
  if (!ensure_rope_s(s, ax.length)) return false;
  const AxialBuffers buf{s->x,    s->x16,   s->row_inv, s->sumsq, s->wide,
                         s->attn, s->gates, s->d_rope,  s->d_err, s->rope_len};
  const AxialWeights aw{&w.m_qkv, &w.m_out, &w.m_ff1, &w.m_ff2, w.ff1, w.gate_b, w.ff1_b, w.ff2_b};
  return run_axial_block(buf, aw, AxialShape{sh.dim, sh.ff_inner, sh.geglu}, tokens, ax, s->bf16 != 0, s->sm_count,
                         s->stream, stack_hook, s);
}

AxisPlan time_axis_s(const StackShape& sh, int clips, int frames) {
  return AxisPlan{1, frames, sh.bands, clips, clips * sh.bands, frames, 1, frames};
}
AxisPlan band_axis_s(const StackShape& sh, int clips, int frames) {
  return AxisPlan{2, frames, sh.bands, clips, clips * frames, sh.bands, frames, sh.bands};
}

// Row statistics of the band-split output (later ones come from the residual
// GEMMs).  Width 256 uses the bundled provider's kernel, so that the stack at
// the bundled sizes reproduces vocalarc_b200_separate bit for bit.
bool row_stats_s(Stack* s, long long tokens) {
  const cudaError_t e =
      s->shape.dim == 256
          ? launch_row_stats(s->x, tokens, s->x16, s->row_inv, s->bf16 != 0, 0, 0, s->stream)
          : launch_row_stats_dim(s->x, tokens, s->shape.dim, s->x16, s->row_inv, s->bf16 != 0, s->stream);
  return slaunched(s, e, "row stats");
}

// Final RMSNorm (gamma folded into mask layer 1) and the per-band mask MLPs;
// x16 / row_inv describe the final x.  Writes the frame-major mask.
bool run_mask_s(Stack* s, int clips, int frames, float* mask_out) {
  const StackShape& sh = s->shape;
  const bool bf = s->bf16 != 0;
  const long long tokens = static_cast<long long>(clips) * sh.bands * frames;
  if (!ensure_mask_tiles_s(s, frames)) return false;
  GemmMaps maps;
  if (!map_rows(s, &maps.a, s->x16, tokens, sh.dim, 128)) return false;
  maps.b = s->m_w1;
  maps.c = maps.d = maps.a;
  GemmArgs args;
  memset(&args, 0, sizeof(args));
  args.k_blocks = sh.dim / 64;
  args.tiles = s->d_tiles1;
  args.tiles_per_chunk = s->n_tiles1;
  args.chunk_rows = sh.bands * frames;
  args.num_tiles = s->n_tiles1 * clips;
  args.out = s->wide;
  args.ldo = sh.hidden;
  args.bias = s->b1;
  args.row_inv = s->row_inv;
  args.err = s->d_err;
  args.pos_div = args.pos_mod = 1;
  if (!slaunched(s, launch_gemm(kEpiTanhBand, bf, maps, args, s->sm_count, s->stream), "mask gemm 1")) return false;
  if (!map_rows(s, &maps.a, s->wide, tokens, sh.hidden, 128)) return false;
  maps.b = s->m_w2;
  args.k_blocks = sh.hidden / 64;
  args.tiles = s->d_tiles2;
  args.tiles_per_chunk = s->n_tiles2;
  args.num_tiles = s->n_tiles2 * clips;
  args.b_box16 = 1;
  args.out = mask_out;
  args.ldo = 0;
  args.bias = s->b2;
  args.row_inv = nullptr;
  args.frames = frames;
  args.mask_ref_layout = 0;
  args.bands = sh.bands;
  args.band_first = s->d_band_first;
  args.band_dim = s->d_band_dim;
  return slaunched(s, launch_gemm(kEpiGluMask, bf, maps, args, s->sm_count, s->stream), "mask gemm 2");
}

bool stack_ready(const Stack* s) { return s != nullptr && s->ok; }

bool check_shape(int clips, int length_or_frames) { return clips > 0 && length_or_frames > 0; }

bool front_end(Stack* s, const float* d_audio, int clips, int length, int frames) {
  const SegmentMap map = whole_clip_map(length);
  return slaunched(s, launch_stft(d_audio, map, clips, frames, s->d_window, s->d_twiddle, s->spec, s->stream,
                                  s->shape.hop),
                   "stft") &&
         slaunched(s, launch_band_split(s->spec, clips, frames, s->band_wt, s->band_wt_off, s->band_gamma,
                                        s->band_gamma_off, s->band_bias, s->x, s->stream, s->shape.dim,
                                        s->shape.bands),
                   "band split");
}

bool back_end(Stack* s, const float* spec, const float* mask, int clips, int length, int frames, float* d_out) {
  return slaunched(s, launch_istft_frames(spec, mask, clips, frames, s->d_window, s->d_twiddle, s->frames_buf,
                                          s->stream),
                   "istft") &&
         slaunched(s, launch_overlap_add(s->frames_buf, clips, frames, length, s->d_window, d_out, s->stream,
                                         s->shape.hop),
                   "overlap-add");
}

bool forward_s(Stack* s, const float* d_audio, int clips, int length, float* d_vocals) {
  const StackShape& sh = s->shape;
  const int frames = length / sh.hop + 1;
  const long long tokens = static_cast<long long>(clips) * sh.bands * frames;
  if (tokens > 0x7fffffffLL) return false;   // GEMM row indices are 32-bit
  if (!ensure_tokens_s(s, tokens) || !ensure_frames_s(s, static_cast<long long>(clips) * frames) ||
      !ensure_rope_s(s, frames > sh.bands ? frames : sh.bands))
    return false;
  if (!front_end(s, d_audio, clips, length, frames) || !row_stats_s(s, tokens)) return false;
  for (int l = 0; l < sh.depth; ++l) {
    if (!run_block_s(s, s->blocks[static_cast<size_t>(2 * l)], tokens, time_axis_s(sh, clips, frames))) return false;
    if (!run_block_s(s, s->blocks[static_cast<size_t>(2 * l + 1)], tokens, band_axis_s(sh, clips, frames)))
      return false;
  }
  return run_mask_s(s, clips, frames, s->mask) && back_end(s, s->spec, s->mask, clips, length, frames, d_vocals);
}

bool sync_check(Stack* s, const char* what) {
  if (!sok(s, cudaStreamSynchronize(s->stream), what)) return false;
  int err = 0;
  if (!sok(s, cudaMemcpy(&err, s->d_err, sizeof(int), cudaMemcpyDeviceToHost), what)) return false;
  if (err != 0) {
    fprintf(stderr, "vocalarc-b200 stack: %s: kernel gave up waiting (code %d)\n", what, err);
    cudaMemset(s->d_err, 0, sizeof(int));
    return false;
  }
  return true;
}

void free_stack(Stack* s) {
  if (s == nullptr) return;
  cudaSetDevice(s->device);
  if (s->stream != nullptr) cudaStreamSynchronize(s->stream);
  void* ptrs[] = {s->d_err,   s->d_window, s->d_twiddle, s->d_rope,  s->model_mem, s->d_tiles1,  s->d_tiles2,
                  s->x,       s->x16,      s->row_inv,   s->sumsq,   s->wide,      s->attn,      s->gates,
                  s->spec,    s->mask,     s->frames_buf, s->audio_in, s->audio_out};
  for (void* p : ptrs)
    if (p != nullptr) cudaFree(p);
  for (cudaEvent_t ev : s->event_pool) cudaEventDestroy(ev);
  if (s->trace_base != nullptr) cudaEventDestroy(s->trace_base);
  if (s->stream != nullptr) cudaStreamDestroy(s->stream);
  delete s;
}

}  // namespace

extern "C" {

size_t vocalarc_b200_stack_weight_count(const vocalarc_b200_stack_config* cfg) {
  StackShape sh;
  return shape_of(cfg, sh) ? sh.total : 0;
}

vocalarc_b200_stack* vocalarc_b200_stack_create(int device, const vocalarc_b200_stack_config* cfg,
                                                const float* weights, size_t count) {
  StackShape sh;
  if (!shape_of(cfg, sh) || weights == nullptr || count != sh.total) {
    fprintf(stderr, "vocalarc-b200 stack: unsupported configuration or weight count\n");
    return nullptr;
  }
  Stack* s = new Stack();
  s->shape = sh;
  s->bf16 = cfg->bf16;
  if (!init_stack(s, device) || !load_weights(s, weights)) {
    free_stack(s);
    return nullptr;
  }
  s->ok = 1;
  return s;
}

void vocalarc_b200_stack_destroy(vocalarc_b200_stack* stack) { free_stack(stack); }

int vocalarc_b200_stack_forward_device(vocalarc_b200_stack* s, const float* d_audio, int clips, int length,
                                       float* d_vocals) {
  if (!stack_ready(s) || d_audio == nullptr || d_vocals == nullptr || !check_shape(clips, length)) return 0;
  cudaSetDevice(s->device);
  return forward_s(s, d_audio, clips, length, d_vocals) ? 1 : 0;
}

int vocalarc_b200_stack_separate(vocalarc_b200_stack* s, const float* audio, int clips, int length, float* vocals) {
  if (!stack_ready(s) || audio == nullptr || vocals == nullptr || !check_shape(clips, length)) return 0;
  cudaSetDevice(s->device);
  const long long samples = 2ll * clips * length;
  if (samples > s->ws_audio) {
    s->ws_audio = 0;
    if (!sgrow(s, &s->audio_in, samples * 4, "cudaMalloc(audio)") ||
        !sgrow(s, &s->audio_out, samples * 4, "cudaMalloc(audio)"))
      return 0;
    s->ws_audio = samples;
  }
  if (!sok(s, cudaMemcpyAsync(s->audio_in, audio, samples * 4, cudaMemcpyHostToDevice, s->stream), "H2D audio") ||
      !forward_s(s, s->audio_in, clips, length, s->audio_out) ||
      !sok(s, cudaMemcpyAsync(vocals, s->audio_out, samples * 4, cudaMemcpyDeviceToHost, s->stream), "D2H vocals"))
    return 0;
  return sync_check(s, "stack separate") ? 1 : 0;
}

int vocalarc_b200_stack_stage_stft(vocalarc_b200_stack* s, const float* d_audio, int clips, int length,
                                   float* d_spec) {
  if (!stack_ready(s) || d_audio == nullptr || d_spec == nullptr || !check_shape(clips, length)) return 0;
  cudaSetDevice(s->device);
  const int frames = length / s->shape.hop + 1;
  return slaunched(s, launch_stft(d_audio, whole_clip_map(length), clips, frames, s->d_window, s->d_twiddle, d_spec,
                                  s->stream, s->shape.hop),
                   "stft")
             ? 1
             : 0;
}

int vocalarc_b200_stack_stage_band_split(vocalarc_b200_stack* s, const float* d_spec, int clips, int frames,
                                         float* d_x) {
  if (!stack_ready(s) || d_spec == nullptr || d_x == nullptr || !check_shape(clips, frames)) return 0;
  cudaSetDevice(s->device);
  return slaunched(s, launch_band_split(d_spec, clips, frames, s->band_wt, s->band_wt_off, s->band_gamma,
                                        s->band_gamma_off, s->band_bias, d_x, s->stream, s->shape.dim,
                                        s->shape.bands),
                   "band split")
             ? 1
             : 0;
}

int vocalarc_b200_stack_stage_block(vocalarc_b200_stack* s, float* d_x, int clips, int frames, int layer, int axis) {
  if (!stack_ready(s) || d_x == nullptr || !check_shape(clips, frames) || layer < 0 || layer >= s->shape.depth ||
      (axis != 0 && axis != 1))
    return 0;
  cudaSetDevice(s->device);
  const StackShape& sh = s->shape;
  const long long tokens = static_cast<long long>(clips) * sh.bands * frames;
  if (tokens > 0x7fffffffLL || !ensure_tokens_s(s, tokens)) return 0;
  const size_t bytes = static_cast<size_t>(tokens) * sh.dim * 4;
  if (!sok(s, cudaMemcpyAsync(s->x, d_x, bytes, cudaMemcpyDeviceToDevice, s->stream), "stage copy") ||
      !row_stats_s(s, tokens))
    return 0;
  const AxisPlan ax = axis == 0 ? time_axis_s(sh, clips, frames) : band_axis_s(sh, clips, frames);
  if (!run_block_s(s, s->blocks[static_cast<size_t>(2 * layer + axis)], tokens, ax)) return 0;
  return sok(s, cudaMemcpyAsync(d_x, s->x, bytes, cudaMemcpyDeviceToDevice, s->stream), "stage copy") ? 1 : 0;
}

int vocalarc_b200_stack_stage_mask(vocalarc_b200_stack* s, const float* d_x, int clips, int frames, float* d_mask) {
  if (!stack_ready(s) || d_x == nullptr || d_mask == nullptr || !check_shape(clips, frames)) return 0;
  cudaSetDevice(s->device);
  const StackShape& sh = s->shape;
  const long long tokens = static_cast<long long>(clips) * sh.bands * frames;
  if (tokens > 0x7fffffffLL || !ensure_tokens_s(s, tokens)) return 0;
  const size_t bytes = static_cast<size_t>(tokens) * sh.dim * 4;
  return sok(s, cudaMemcpyAsync(s->x, d_x, bytes, cudaMemcpyDeviceToDevice, s->stream), "stage copy") &&
                 row_stats_s(s, tokens) && run_mask_s(s, clips, frames, d_mask)
             ? 1
             : 0;
}

int vocalarc_b200_stack_stage_istft(vocalarc_b200_stack* s, const float* d_spec, const float* d_mask, int clips,
                                    int length, float* d_audio) {
  if (!stack_ready(s) || d_spec == nullptr || d_mask == nullptr || d_audio == nullptr || !check_shape(clips, length))
    return 0;
  cudaSetDevice(s->device);
  const int frames = length / s->shape.hop + 1;
  if (!ensure_frames_s(s, static_cast<long long>(clips) * frames)) return 0;
  return back_end(s, d_spec, d_mask, clips, length, frames, d_audio) ? 1 : 0;
}

int vocalarc_b200_stack_synchronize(vocalarc_b200_stack* s) {
  if (!stack_ready(s)) return 0;
  cudaSetDevice(s->device);
  return sync_check(s, "stack synchronize") ? 1 : 0;
}

void* vocalarc_b200_stack_stream(vocalarc_b200_stack* s) { return stack_ready(s) ? s->stream : nullptr; }

int vocalarc_b200_stack_take_device_error(vocalarc_b200_stack* s) {
  if (s == nullptr || s->d_err == nullptr) return 0;
  cudaSetDevice(s->device);
  int err = 0;
  cudaMemcpy(&err, s->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  cudaMemset(s->d_err, 0, sizeof(int));
  return err;
}

long long vocalarc_b200_stack_launch_count(const vocalarc_b200_stack* s) { return s != nullptr ? s->launches : 0; }

int vocalarc_b200_stack_trace_begin(vocalarc_b200_stack* s) {
  if (!stack_ready(s)) return 0;
  cudaSetDevice(s->device);
  if (s->trace_base == nullptr && cudaEventCreate(&s->trace_base) != cudaSuccess) return 0;
  s->trace_entries.clear();
  cudaEventRecord(s->trace_base, s->stream);
  s->trace = 1;
  return 1;
}

int vocalarc_b200_stack_trace_end(vocalarc_b200_stack* s, char* out, int capacity) {
  if (!stack_ready(s) || !s->trace || out == nullptr || capacity <= 0) return 0;
  cudaSetDevice(s->device);
  s->trace = 0;
  if (!sok(s, cudaStreamSynchronize(s->stream), "trace")) return 0;
  std::vector<std::string> names;
  std::vector<double> ms;
  std::vector<long long> counts;
  cudaEvent_t prev = s->trace_base;
  for (auto& entry : s->trace_entries) {
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
  s->trace_entries.clear();
  std::string text;
  char line[256];
  for (size_t i = 0; i < names.size(); ++i) {
    snprintf(line, sizeof(line), "%s\t%lld\t%.6f\n", names[i].c_str(), counts[i], ms[i]);
    text += line;
  }
  snprintf(out, static_cast<size_t>(capacity), "%s", text.c_str());
  return 1;
}

}  // extern "C"
