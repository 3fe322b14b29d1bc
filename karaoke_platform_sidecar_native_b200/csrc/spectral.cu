// Spectral front/back end and memory-bound kernels of the separation forward.
//
//  * stft_kernel: center=True framing with reflect padding, periodic Hann
//    window, 2048-point real FFT through a 1024-point complex FFT in shared
//    memory (stft_channels, native/vocalarc_separation.c:1044-1064).  The
//    reference FFT runs in double on the host; this one is fp32 with
//    double-precision twiddles, checked against the oracle by SNR.
//  * band_split_kernel: per band gather + RMSNorm + Linear(d_b -> 256) + bias
//    (band_split_one :887-915), fp32 SIMT; writes the band-major token layout.
//  * row_stats_kernel: 16-bit copy of the residual and its per-row RMSNorm
//    factor for the norm-folded GEMMs (rms_norm_row :419-424).
//  * istft_frames_kernel / overlap_add_kernel: complex mask, Hermitian
//    inverse real FFT, window, overlap-add in frame order, divide by the
//    window envelope or 0 when it is <= 1e-12 (istft_channels :1084-1127).
//  * demix_kernel: chunk overlap-add with the linear fade and first/final
//    batch rule, divide by the weight sum, crop the border
//    (Separator::demix onnx/native/onnx_sidecar.cpp:725-782).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "ptx.cuh"
#include "vab_internal.h"

namespace vab {

namespace {

__device__ __forceinline__ int reflect_index(int index, int length) {
  // Repeated reflection about 0 and length-1 (vocalarc_separation.c:1027-1034).
  if (length <= 1) return 0;
  const int period = 2 * length - 2;
  int r = index % period;
  if (r < 0) r += period;
  return r >= length ? period - r : r;
}

// Sample i (0 <= i < seg_length) of channel ch of segment c.
__device__ __forceinline__ float segment_sample(const float* audio, const SegmentMap& m, int c, int ch, int i) {
  if (m.mode == 0) return audio[c * m.clip_stride + static_cast<long long>(ch) * m.clip_length + i];
  const int start = (m.first_chunk + c) * m.step;
  const int available = start < m.padded ? min(m.seg_length, m.padded - start) : 0;
  int j;
  if (i < available) {
    j = start + i;
  } else if (available > m.seg_length / 2 && available > 1) {
    j = start + reflect_index(i, available);   // pad_chunk, onnx_sidecar.cpp:366-383
  } else {
    return 0.0f;
  }
  const int src = m.border > 0 ? reflect_index(j - m.border, m.clip_length) : j;
  return audio[static_cast<long long>(ch) * m.clip_length + src];
}

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
  return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// Two in-place 1024-point radix-2 decimation-in-frequency FFTs (forward,
// e^{-2 pi i k n / 1024}); the result lands in bit-reversed order.
// tw[k] = e^{-2 pi i k / 2048}, so the 1024-point twiddle W^k is tw[2k].
__device__ void fft1024_pair(float2* buf0, float2* buf1, const float2* tw) {
  for (int span = 512, log_span = 9; span >= 1; span >>= 1, --log_span) {
    for (int b = threadIdx.x; b < 1024; b += blockDim.x) {
      float2* buf = b < 512 ? buf0 : buf1;
      const int bb = b & 511;
      const int pos = bb & (span - 1);
      const int i = ((bb >> log_span) << (log_span + 1)) + pos;
      const int j = i + span;
      const float2 a = buf[i];
      const float2 c = buf[j];
      buf[i] = make_float2(a.x + c.x, a.y + c.y);
      const float2 w = tw[(pos << (9 - log_span)) * 2];
      buf[j] = cmul(make_float2(a.x - c.x, a.y - c.y), w);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ int brev10(int x) { return static_cast<int>(__brev(static_cast<unsigned>(x)) >> 22); }

__global__ void __launch_bounds__(256) stft_kernel(const float* __restrict__ audio, SegmentMap map, int frames,
                                                   const float* __restrict__ window,
                                                   const float2* __restrict__ twiddle, float* __restrict__ spec) {
  __shared__ float2 buf[2][1024];
  __shared__ float2 tw[1025];
  const int f = blockIdx.x;
  const int c = blockIdx.y;
  for (int k = threadIdx.x; k < 1025; k += blockDim.x) tw[k] = twiddle[k];
  const int start = f * kHop - kNfft / 2;
  for (int n = threadIdx.x; n < kNfft; n += blockDim.x) {
    const int s = reflect_index(start + n, map.seg_length);
    const float w = window[n];
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const float x = segment_sample(audio, map, c, ch, s) * w;
      float* slot = reinterpret_cast<float*>(&buf[ch][n >> 1]);
      slot[n & 1] = x;
    }
  }
  __syncthreads();
  fft1024_pair(buf[0], buf[1], tw);
  // X[k] = E[k] + W^k O[k],  E = (Z[k] + conj Z[1024-k]) / 2,  O = (Z[k] - conj Z[1024-k]) / (2i).
  float4* out = reinterpret_cast<float4*>(spec) + (static_cast<long long>(c) * frames + f) * kFreqBins;
  for (int k = threadIdx.x; k < kFreqBins; k += blockDim.x) {
    float v[4];
    const float2 w = tw[k];
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const float2 zk = buf[ch][brev10(k & 1023)];
      const float2 zr = buf[ch][brev10((1024 - k) & 1023)];
      const float2 e = make_float2(0.5f * (zk.x + zr.x), 0.5f * (zk.y - zr.y));
      const float2 o = make_float2(0.5f * (zk.y + zr.y), -0.5f * (zk.x - zr.x));
      const float2 x = make_float2(e.x + (w.x * o.x - w.y * o.y), e.y + (w.x * o.y + w.y * o.x));
      v[2 * ch] = x.x;
      v[2 * ch + 1] = x.y;
    }
    out[k] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// ---------------------------------------------------------------- band split
constexpr int kBandFrames = 32;

__global__ void __launch_bounds__(256) band_split_kernel(const float* __restrict__ spec, int frames,
                                                         const float* __restrict__ band_wt,
                                                         const long long* __restrict__ band_wt_offset,
                                                         const float* __restrict__ band_gamma,
                                                         const int* __restrict__ band_gamma_offset,
                                                         const float* __restrict__ band_bias, float* __restrict__ x) {
  extern __shared__ float rows[];  // [kBandFrames][d]
  const int t0 = blockIdx.x * kBandFrames;
  const int band = blockIdx.y;
  const int c = blockIdx.z;
  const int goff = band_gamma_offset[band];
  const int d = band_gamma_offset[band + 1] - goff;
  const int first = goff / 4;  // the gamma table is laid out in bin order: offset = 4 * first bin
  const float* gamma = band_gamma + goff;
  for (int idx = threadIdx.x; idx < kBandFrames * d; idx += blockDim.x) {
    const int tt = idx / d;
    const int k = idx - tt * d;
    const int t = t0 + tt;
    rows[idx] = t < frames ? spec[((static_cast<long long>(c) * frames + t) * kFreqBins + first) * 4 + k] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int tt = warp; tt < kBandFrames; tt += 8) {
    float* row = rows + tt * d;
    float ss = 0.f;
    for (int k = lane; k < d; k += 32) ss += row[k] * row[k];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    const float inv = sqrtf(static_cast<float>(d)) / sqrtf(ss + 1.0e-12f);
    for (int k = lane; k < d; k += 32) row[k] = row[k] * inv * gamma[k];
  }
  __syncthreads();
  const int n = threadIdx.x;
  const float* wt = band_wt + band_wt_offset[band];  // [d][256]
  float acc[kBandFrames];
  const float b = band_bias[band * kDim + n];
#pragma unroll
  for (int tt = 0; tt < kBandFrames; ++tt) acc[tt] = b;
  for (int k = 0; k < d; k += 4) {
    const float w0 = __ldg(wt + (k + 0) * kDim + n);
    const float w1 = __ldg(wt + (k + 1) * kDim + n);
    const float w2 = __ldg(wt + (k + 2) * kDim + n);
    const float w3 = __ldg(wt + (k + 3) * kDim + n);
#pragma unroll
    for (int tt = 0; tt < kBandFrames; ++tt) {
      const float4 r = *reinterpret_cast<const float4*>(rows + tt * d + k);
      acc[tt] = fmaf(r.x, w0, acc[tt]);
      acc[tt] = fmaf(r.y, w1, acc[tt]);
      acc[tt] = fmaf(r.z, w2, acc[tt]);
      acc[tt] = fmaf(r.w, w3, acc[tt]);
    }
  }
  float* out = x + ((static_cast<long long>(c) * kBands + band) * frames) * kDim + n;
#pragma unroll
  for (int tt = 0; tt < kBandFrames; ++tt)
    if (t0 + tt < frames) out[static_cast<long long>(t0 + tt) * kDim] = acc[tt];
}

// ---------------------------------------------------------------- row statistics
// x16 = 16-bit copy of x, inv = sqrt(256) / sqrt(sum x^2 + 1e-12) per row (the
// scale of rms_norm_row_scalar, vocalarc_separation.c:419-424; the gamma is
// folded into the consuming GEMM's weights).  One warp per 256-wide row.
template <typename T>
__global__ void __launch_bounds__(256) row_stats_kernel(const float* __restrict__ x, long long rows,
                                                        T* __restrict__ x16, float* __restrict__ inv, int remap_s0,
                                                        int remap_l0) {
  const long long r = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const float4* src = reinterpret_cast<const float4*>(x + r * kDim);
  const float4 a = src[lane];
  const float4 b = src[32 + lane];
  float ss = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  // Optional remap of the token order: physical [s0][l0] -> [l0][s0].
  long long out_row = r;
  if (remap_s0 > 0) out_row = (r % remap_l0) * remap_s0 + r / remap_l0;
  T* dst = x16 + out_row * kDim;
  uint2 p0, p1;
  p0.x = ElemTraits<T>::pack2(a.x, a.y);
  p0.y = ElemTraits<T>::pack2(a.z, a.w);
  p1.x = ElemTraits<T>::pack2(b.x, b.y);
  p1.y = ElemTraits<T>::pack2(b.z, b.w);
  *reinterpret_cast<uint2*>(dst + lane * 4) = p0;
  *reinterpret_cast<uint2*>(dst + 128 + lane * 4) = p1;
  if (lane == 0) inv[out_row] = 16.0f / sqrtf(ss + 1.0e-12f);   // sqrtf(256) / sqrtf(sum + 1e-12)
}

// ---------------------------------------------------------------- iSTFT
__global__ void __launch_bounds__(256) istft_frames_kernel(const float* __restrict__ spec,
                                                           const float* __restrict__ mask, int frames,
                                                           const float* __restrict__ window,
                                                           const float2* __restrict__ twiddle,
                                                           float* __restrict__ frames_out) {
  __shared__ float2 y[2][kFreqBins];
  __shared__ float2 buf[2][1024];
  __shared__ float2 tw[1025];
  const int f = blockIdx.x;
  const int c = blockIdx.y;
  for (int k = threadIdx.x; k < 1025; k += blockDim.x) tw[k] = twiddle[k];
  const long long base = (static_cast<long long>(c) * frames + f) * kFreqBins;
  const float4* s4 = reinterpret_cast<const float4*>(spec) + base;
  const float4* m4 = reinterpret_cast<const float4*>(mask) + base;
  for (int k = threadIdx.x; k < kFreqBins; k += blockDim.x) {
    const float4 s = s4[k];
    const float4 m = m4[k];
    float2 y0 = make_float2(s.x * m.x - s.y * m.y, s.x * m.y + s.y * m.x);
    float2 y1 = make_float2(s.z * m.z - s.w * m.w, s.z * m.w + s.w * m.z);
    if (k == 0 || k == 1024) {  // the real part of the inverse ignores these imaginary parts
      y0.y = 0.f;
      y1.y = 0.f;
    }
    y[0][k] = y0;
    y[1][k] = y1;
  }
  __syncthreads();
  // Z[k] = (X[k] + conj X[1024-k]) + i e^{+2 pi i k / 2048} (X[k] - conj X[1024-k]); store conj(Z)
  // so that a forward FFT followed by conjugation gives the inverse.
  for (int k = threadIdx.x; k < 1024; k += blockDim.x) {
    const float2 e = make_float2(tw[k].x, -tw[k].y);
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const float2 a = y[ch][k];
      const float2 b = y[ch][1024 - k];
      const float2 sum = make_float2(a.x + b.x, a.y - b.y);
      const float2 dif = make_float2(a.x - b.x, a.y + b.y);
      const float2 ed = cmul(e, dif);
      const float2 z = make_float2(sum.x - ed.y, sum.y + ed.x);
      buf[ch][k] = make_float2(z.x, -z.y);
    }
  }
  __syncthreads();
  fft1024_pair(buf[0], buf[1], tw);
  const float scale = 1.0f / 2048.0f;
  for (int m = threadIdx.x; m < 1024; m += blockDim.x) {
    const float w0 = window[2 * m], w1 = window[2 * m + 1];
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const float2 z = buf[ch][brev10(m)];
      float2* dst = reinterpret_cast<float2*>(frames_out + ((static_cast<long long>(c) * 2 + ch) * frames + f) * kNfft);
      dst[m] = make_float2(z.x * scale * w0, -z.y * scale * w1);
    }
  }
}

__global__ void __launch_bounds__(256) overlap_add_kernel(const float* __restrict__ frames_buf, int frames,
                                                          int seg_length, const float* __restrict__ window,
                                                          float* __restrict__ seg_out) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= seg_length) return;
  const int cc = blockIdx.y;  // segment * 2 + channel
  // Frames f with f*512 - 1024 <= s < f*512 + 1024, i.e. f in [q - 3, q] with
  // q = floor((s + 1024) / 512) (s >= 0, so the division is a floor).
  const int q = (s + kNfft / 2) / kHop;
  const int f_hi = min(frames - 1, q);
  const int f_lo = max(0, q - (kNfft / kHop - 1));
  float acc = 0.f, env = 0.f;
  const float* fb = frames_buf + static_cast<long long>(cc) * frames * kNfft;
  for (int f = f_lo; f <= f_hi; ++f) {
    const int i = s - (f * kHop - kNfft / 2);
    if (i < 0 || i >= kNfft) continue;
    acc += fb[static_cast<long long>(f) * kNfft + i];
    const float w = window[i];
    env += w * w;
  }
  seg_out[static_cast<long long>(cc) * seg_length + s] = env > 1.0e-12f ? acc / env : 0.0f;
}

__global__ void __launch_bounds__(256) demix_kernel(const float* __restrict__ seg_out, SegmentMap map, int chunks,
                                                    int model_batch, float* __restrict__ vocals) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= map.clip_length) return;
  const int ch = blockIdx.y;
  const int chunk = map.seg_length;
  const int fade = chunk / 10;
  const int p = s + map.border;
  const int c_hi = min(chunks - 1, p / map.step);
  int c_lo = (p - chunk) / map.step + 1;
  if (p - chunk < 0) c_lo = 0;
  const int batches = (chunks + model_batch - 1) / model_batch;
  const int final_first = (batches - 1) * model_batch;
  const bool first_forced = model_batch == 1 || chunks == 1;
  float res = 0.f, cnt = 0.f;
  for (int c = max(c_lo, 0); c <= c_hi; ++c) {
    const int start = c * map.step;
    const int valid = min(chunk, map.padded - start);
    const int i = p - start;
    if (i < 0 || i >= valid) continue;
    float w = 1.0f;
    const bool forced = (c == 0 && first_forced) || c >= final_first;
    if (!forced && i >= chunk - fade) w = 1.0f - static_cast<float>(i - (chunk - fade)) / static_cast<float>(fade);
    res += seg_out[(static_cast<long long>(c) * 2 + ch) * chunk + i] * w;
    cnt += w;
  }
  vocals[static_cast<long long>(ch) * map.clip_length + s] = res / fmaxf(cnt, 1.0e-12f);
}

__global__ void transpose_tokens_kernel(const float* __restrict__ src, float* __restrict__ dst, int s0, int l0) {
  // [s0][l0][256] -> [l0][s0][256]; one warp-row of 256 floats per block row.
  const long long token = blockIdx.x;
  const int s = static_cast<int>(token / l0);
  const int l = static_cast<int>(token % l0);
  const float4* a = reinterpret_cast<const float4*>(src + token * kDim);
  float4* b = reinterpret_cast<float4*>(dst + (static_cast<long long>(l) * s0 + s) * kDim);
  b[threadIdx.x] = a[threadIdx.x];
}

// Demix over a contiguous chunk range [c0, c1) of the track (sharding of one
// track across GPUs).  The accumulators of padded sample p start from `init`
// (the previous range's partial sums for its seam, or zero) and add this
// range's chunks in ascending order -- the summation order of demix_kernel, so
// the sharded result is bit-identical to the single-GPU demix.  With seam_out
// set the partial sums (channel 0, channel 1, weight) are written instead of
// the divided, cropped output.
__global__ void __launch_bounds__(256) demix_range_kernel(const float* __restrict__ seg_out, SegmentMap map,
                                                          int chunks, int model_batch, DemixRange r) {
  const int p = r.p0 + static_cast<int>(blockIdx.x * blockDim.x + threadIdx.x);
  if (p >= r.p1) return;
  const int chunk = map.seg_length;
  const int fade = chunk / 10;
  const int c_hi = min(chunks - 1, p / map.step);
  int c_lo = (p - chunk) / map.step + 1;
  if (p - chunk < 0) c_lo = 0;
  const int batches = (chunks + model_batch - 1) / model_batch;
  const int final_first = (batches - 1) * model_batch;
  const bool first_forced = model_batch == 1 || chunks == 1;
  float res0 = 0.f, res1 = 0.f, cnt = 0.f;
  const int k = p - r.init_p0;
  if (r.init != nullptr && k >= 0 && k < r.init_len) {
    res0 = r.init[k];
    res1 = r.init[r.init_len + k];
    cnt = r.init[2 * r.init_len + k];
  }
  for (int c = max(c_lo, r.c0); c <= min(c_hi, r.c1 - 1); ++c) {
    const int start = c * map.step;
    const int valid = min(chunk, map.padded - start);
    const int i = p - start;
    if (i < 0 || i >= valid) continue;
    float w = 1.0f;
    const bool forced = (c == 0 && first_forced) || c >= final_first;
    if (!forced && i >= chunk - fade) w = 1.0f - static_cast<float>(i - (chunk - fade)) / static_cast<float>(fade);
    const float* o = seg_out + static_cast<long long>(c - r.c0) * 2 * chunk;
    res0 += o[i] * w;
    res1 += o[chunk + i] * w;
    cnt += w;
  }
  if (r.seam_out != nullptr) {
    const int len = r.p1 - r.p0;
    const int j = p - r.p0;
    r.seam_out[j] = res0;
    r.seam_out[len + j] = res1;
    r.seam_out[2 * len + j] = cnt;
  } else {
    const int s = p - map.border;
    if (s >= 0 && s < map.clip_length) {
      r.vocals[s] = res0 / fmaxf(cnt, 1.0e-12f);
      r.vocals[static_cast<long long>(map.clip_length) + s] = res1 / fmaxf(cnt, 1.0e-12f);
    }
  }
}

// ---------------------------------------------------------------- bigshifts + TTA
// Separator::separate / bigshift of the ONNX sidecar (onnx_sidecar.cpp:556-575,
// :784-790, rotate/unrotate/scale/add :385-421).  Variant v of the mix (0: as
// is, 1: channels swapped, 2: polarity flipped) rotated by shift k of B:
// out[v][k][ch][i] = sign_v * mix[ch_v][(n - shift_k + i) % n].
__global__ void __launch_bounds__(256) tta_inputs_kernel(const float* __restrict__ mix, int n, int shifts,
                                                         int variants, float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int vk = blockIdx.y;   // v * shifts + k
  const int v = vk / shifts, k = vk - v * shifts;
  const int shift = static_cast<int>((static_cast<long long>(k) * (n / shifts)) % n);
  const int src = static_cast<int>((static_cast<long long>(n) - shift + i) % n);
#pragma unroll
  for (int ch = 0; ch < 2; ++ch) {
    const int ch_src = v == 1 ? 1 - ch : ch;
    float x = mix[static_cast<long long>(ch_src) * n + src];
    if (v == 2) x *= -1.0f;
    out[(static_cast<long long>(vk) * 2 + ch) * n + i] = x;
  }
}

// Combines the estimates est[v][k][2][n] in the reference's float order:
// bigshift r_v = (0 + e_0 + e_1 + ...) * (1/B) with e_k rotated back; without
// TTA the result is r_0, with TTA ((r_0 + swap(r_1)) + (-1) * (-1 * r_2)) * (1/3).
__global__ void __launch_bounds__(256) tta_combine_kernel(const float* __restrict__ est, int n, int shifts,
                                                          int tta, float* __restrict__ vocals) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int ch = blockIdx.y;
  const float inv_shifts = 1.0f / static_cast<float>(shifts);
  float r[3];
  for (int v = 0; v < (tta ? 3 : 1); ++v) {
    const int ch_v = v == 1 ? 1 - ch : ch;   // the swapped estimate is swapped back
    float acc = 0.0f;
    for (int k = 0; k < shifts; ++k) {
      const int shift = static_cast<int>((static_cast<long long>(k) * (n / shifts)) % n);
      const int src = static_cast<int>((static_cast<long long>(i) + shift) % n);
      acc = __fadd_rn(acc, est[((static_cast<long long>(v) * shifts + k) * 2 + ch_v) * n + src]);
    }
    r[v] = __fmul_rn(acc, inv_shifts);
  }
  float out = r[0];
  if (tta) {
    const float inverted = __fmul_rn(r[2], -1.0f);
    const float total = __fadd_rn(r[0], r[1]);
    out = __fmul_rn(__fadd_rn(total, __fmul_rn(-1.0f, inverted)), 1.0f / 3.0f);
  }
  vocals[static_cast<long long>(ch) * n + i] = out;
}

}  // namespace

cudaError_t launch_stft(const float* audio, SegmentMap map, int segments, int frames, const float* window,
                        const float2* twiddle, float* spec, cudaStream_t stream) {
  if (segments <= 0 || frames <= 0) return cudaSuccess;
  stft_kernel<<<dim3(frames, segments), 256, 0, stream>>>(audio, map, frames, window, twiddle, spec);
  return cudaGetLastError();
}

cudaError_t launch_band_split(const float* spec, int segments, int frames, const float* band_wt,
                              const long long* band_wt_offset, const float* band_gamma, const int* band_gamma_offset,
                              const float* band_bias, float* x, cudaStream_t stream) {
  static bool configured = false;
  const int smem = kBandFrames * 516 * 4;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(band_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((frames + kBandFrames - 1) / kBandFrames, kBands, segments);
  band_split_kernel<<<grid, 256, smem, stream>>>(spec, frames, band_wt, band_wt_offset, band_gamma,
                                                  band_gamma_offset, band_bias, x);
  return cudaGetLastError();
}

cudaError_t launch_row_stats(const float* x, long long rows, void* x16, float* inv, bool bf16, int remap_s0,
                             int remap_l0, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const long long blocks = (rows + 7) / 8;
  if (bf16)
    row_stats_kernel<__nv_bfloat16><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        x, rows, static_cast<__nv_bfloat16*>(x16), inv, remap_s0, remap_l0);
  else
    row_stats_kernel<__half><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        x, rows, static_cast<__half*>(x16), inv, remap_s0, remap_l0);
  return cudaGetLastError();
}

cudaError_t launch_istft_frames(const float* spec, const float* mask, int segments, int frames, const float* window,
                                const float2* twiddle, float* frames_out, cudaStream_t stream) {
  if (segments <= 0 || frames <= 0) return cudaSuccess;
  istft_frames_kernel<<<dim3(frames, segments), 256, 0, stream>>>(spec, mask, frames, window, twiddle, frames_out);
  return cudaGetLastError();
}

cudaError_t launch_overlap_add(const float* frames_buf, int segments, int frames, int seg_length, const float* window,
                               float* seg_out, cudaStream_t stream) {
  if (segments <= 0 || seg_length <= 0) return cudaSuccess;
  dim3 grid((seg_length + 255) / 256, segments * 2);
  overlap_add_kernel<<<grid, 256, 0, stream>>>(frames_buf, frames, seg_length, window, seg_out);
  return cudaGetLastError();
}

cudaError_t launch_demix(const float* seg_out, SegmentMap map, int chunks, int model_batch, float* vocals,
                         cudaStream_t stream) {
  if (map.clip_length <= 0) return cudaSuccess;
  dim3 grid((map.clip_length + 255) / 256, 2);
  demix_kernel<<<grid, 256, 0, stream>>>(seg_out, map, chunks, model_batch, vocals);
  return cudaGetLastError();
}

cudaError_t launch_demix_range(const float* seg_out, SegmentMap map, int chunks, int model_batch,
                               const DemixRange& range, cudaStream_t stream) {
  if (range.p1 <= range.p0) return cudaSuccess;
  demix_range_kernel<<<(range.p1 - range.p0 + 255) / 256, 256, 0, stream>>>(seg_out, map, chunks, model_batch, range);
  return cudaGetLastError();
}

cudaError_t launch_tta_inputs(const float* mix, int n, int shifts, int variants, float* out, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  tta_inputs_kernel<<<dim3((n + 255) / 256, shifts * variants), 256, 0, stream>>>(mix, n, shifts, variants, out);
  return cudaGetLastError();
}

cudaError_t launch_tta_combine(const float* est, int n, int shifts, int tta, float* vocals, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  tta_combine_kernel<<<dim3((n + 255) / 256, 2), 256, 0, stream>>>(est, n, shifts, tta, vocals);
  return cudaGetLastError();
}

cudaError_t launch_transpose_tokens(const float* src, float* dst, int s0, int l0, cudaStream_t stream) {
  const long long tokens = static_cast<long long>(s0) * l0;
  if (tokens <= 0) return cudaSuccess;
  transpose_tokens_kernel<<<static_cast<unsigned>(tokens), 64, 0, stream>>>(src, dst, s0, l0);
  return cudaGetLastError();
}

}  // namespace vab
