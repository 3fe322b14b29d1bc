// Spectral front/back end and memory-bound kernels of the separation forward.
//
//  * stft_kernel: center=True framing with reflect padding, periodic Hann
//    window, 2048-point real FFT through a 1024-point complex FFT done as a
//    four-step 32 x 32 transform in registers, one warp per frame and channel
//    (stft_channels, native/vocalarc_separation.c:1044-1064).  The
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


// ---------------------------------------------------------------- STFT
// One warp per (frame, channel), four frames per CTA.  The 2048-point real FFT
// is a 1024-point complex FFT of z[n] = x[2n] + i x[2n+1] done as a four-step
// 32 x 32 transform with n = 32 n1 + n2, k = k1 + 32 k2: lane n2 holds
// z[32 n1 + n2] for all n1 in registers, runs a 32-point FFT over n1, applies
// W_1024^(n2 k1), the warp transposes through shared memory, and lane k1 runs
// the second 32-point FFT over n2, giving Z[k1 + 32 k2].  Then
// X[k] = E[k] + W_2048^k O[k] from Z[k] and Z[1024 - k].  tw[k] = e^{-2 pi i k / 2048}.
constexpr int kStftFramesPerCta = 4;
constexpr int kStftTw = 1028;   // twiddle table entries kept in shared memory (1025 used)
constexpr int kStftBuf = 32 * 33;   // one warp's padded 32 x 32 transpose buffer (float2)
constexpr int kStftSmem = (kStftTw + 2 * kStftFramesPerCta * kStftBuf) * 8;

__host__ __device__ constexpr int brev5(int i) {
  return ((i & 1) << 4) | ((i & 2) << 2) | (i & 4) | ((i & 8) >> 2) | ((i & 16) >> 4);
}

// e^{-2 pi i k / 2048} for 0 <= k < 2048 from the half table.
__device__ __forceinline__ float2 tw2048(const float2* tw, int k) {
  const float2 w = tw[k <= 1024 ? k : k - 1024];
  return k <= 1024 ? w : make_float2(-w.x, -w.y);
}

// One radix-2 decimation-in-time stage of span M over 32 registers.
template <int M>
__device__ __forceinline__ void fft32_stage(float2 (&b)[32], const float2* tw) {
  constexpr int kHalf = M / 2;
#pragma unroll
  for (int k = 0; k < 32; k += M) {
#pragma unroll
    for (int j = 0; j < kHalf; ++j) {
      const float2 u = b[k + j];
      float2 t = b[k + j + kHalf];
      if (j != 0) t = cmul(t, tw[64 * j * (32 / M)]);
      b[k + j] = make_float2(u.x + t.x, u.y + t.y);
      b[k + j + kHalf] = make_float2(u.x - t.x, u.y - t.y);
    }
  }
}

// In-register radix-2 decimation-in-time 32-point FFT (forward), natural
// order in and out; every index is a compile-time constant.
__device__ __forceinline__ void fft32(float2 (&a)[32], const float2* tw) {
  float2 b[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) b[i] = a[brev5(i)];
  fft32_stage<2>(b, tw);
  fft32_stage<4>(b, tw);
  fft32_stage<8>(b, tw);
  fft32_stage<16>(b, tw);
  fft32_stage<32>(b, tw);
#pragma unroll
  for (int i = 0; i < 32; ++i) a[i] = b[i];
}

__global__ void __launch_bounds__(256, 3) stft_kernel(const float* __restrict__ audio, SegmentMap map, int frames,
                                                   int hop, const float* __restrict__ window,
                                                   const float2* __restrict__ twiddle, float* __restrict__ spec) {
  extern __shared__ float2 stft_smem[];
  float2* tw = stft_smem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float2* buf = stft_smem + kStftTw + warp * kStftBuf;
  for (int k = threadIdx.x; k < 1025; k += blockDim.x) tw[k] = twiddle[k];
  const int f = blockIdx.x * kStftFramesPerCta + (warp >> 1);
  const int ch = warp & 1;
  const int c = blockIdx.y;
  const bool active = f < frames;   // warp-uniform; inactive warps only help load the table
  const int start = f * hop - kNfft / 2;
  // Contiguous source run for frames that need no reflection (warp-uniform).
  long long base = -1;
  if (active && start >= 0 && start + kNfft <= map.seg_length) {
    if (map.mode == 0) {
      base = c * map.clip_stride + static_cast<long long>(ch) * map.clip_length + start;
    } else {
      const int cs = (map.first_chunk + c) * map.step;
      const int available = cs < map.padded ? min(map.seg_length, map.padded - cs) : 0;
      if (start + kNfft <= available) {
        const int j0 = cs + start - map.border;
        if (j0 >= 0 && j0 + kNfft <= map.clip_length) base = static_cast<long long>(ch) * map.clip_length + j0;
      }
    }
  }
  float2 a[32];
#pragma unroll
  for (int n1 = 0; n1 < 32; ++n1) {
    const int n = 64 * n1 + 2 * lane;
    const float2 w = *reinterpret_cast<const float2*>(window + n);
    float x0 = 0.f, x1 = 0.f;
    if (!active) {
    } else if (base >= 0) {
      x0 = __ldg(audio + base + n);
      x1 = __ldg(audio + base + n + 1);
    } else {
      x0 = segment_sample(audio, map, c, ch, reflect_index(start + n, map.seg_length));
      x1 = segment_sample(audio, map, c, ch, reflect_index(start + n + 1, map.seg_length));
    }
    a[n1] = make_float2(x0 * w.x, x1 * w.y);
  }
  // The sample loads above are in flight while the table copy completes.
  __syncthreads();
  if (!active) return;
  fft32(a, tw);   // a[k1] for this n2 = lane
#pragma unroll
  for (int k1 = 1; k1 < 32; ++k1) a[k1] = cmul(a[k1], tw2048(tw, 2 * ((lane * k1) & 1023)));
#pragma unroll
  for (int k1 = 0; k1 < 32; ++k1) buf[k1 * 33 + lane] = a[k1];
  __syncwarp();
#pragma unroll
  for (int n2 = 0; n2 < 32; ++n2) a[n2] = buf[lane * 33 + n2];
  __syncwarp();
  fft32(a, tw);   // a[k2] = Z[lane + 32 k2]
#pragma unroll
  for (int k2 = 0; k2 < 32; ++k2) buf[k2 * 33 + lane] = a[k2];
  __syncwarp();
  // X[k] = E[k] + W^k O[k],  E = (Z[k] + conj Z[1024-k]) / 2,  O = (Z[k] - conj Z[1024-k]) / (2i).
  float* out = spec + (static_cast<long long>(c) * frames + f) * kFreqBins * 4 + 2 * ch;
  for (int k = lane; k < kFreqBins; k += 32) {
    const int kk = k & 1023, kr = (1024 - k) & 1023;
    const float2 zk = buf[(kk >> 5) * 33 + (kk & 31)];
    const float2 zr = buf[(kr >> 5) * 33 + (kr & 31)];
    const float2 w = tw[k];
    const float2 e = make_float2(0.5f * (zk.x + zr.x), 0.5f * (zk.y - zr.y));
    const float2 o = make_float2(0.5f * (zk.y + zr.y), -0.5f * (zk.x - zr.x));
    *reinterpret_cast<float2*>(out + static_cast<long long>(k) * 4) =
        make_float2(e.x + (w.x * o.x - w.y * o.y), e.y + (w.x * o.y + w.y * o.x));
  }
}

// ---------------------------------------------------------------- band split
// One CTA per (32 frames, band, segment), one thread per output column
// (DIM = 256 for the bundled model, 512 for a dim-512 stack); the band count
// is gridDim.y.
constexpr int kBandFrames = 32;

template <int DIM>
__global__ void __launch_bounds__(DIM) band_split_kernel(const float* __restrict__ spec, int frames,
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
  for (int tt = warp; tt < kBandFrames; tt += DIM / 32) {
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
  const float* wt = band_wt + band_wt_offset[band];  // [d][DIM]
  float acc[kBandFrames];
  const float b = band_bias[band * DIM + n];
#pragma unroll
  for (int tt = 0; tt < kBandFrames; ++tt) acc[tt] = b;
  for (int k = 0; k < d; k += 4) {
    const float w0 = __ldg(wt + (k + 0) * DIM + n);
    const float w1 = __ldg(wt + (k + 1) * DIM + n);
    const float w2 = __ldg(wt + (k + 2) * DIM + n);
    const float w3 = __ldg(wt + (k + 3) * DIM + n);
#pragma unroll
    for (int tt = 0; tt < kBandFrames; ++tt) {
      const float4 r = *reinterpret_cast<const float4*>(rows + tt * d + k);
      acc[tt] = fmaf(r.x, w0, acc[tt]);
      acc[tt] = fmaf(r.y, w1, acc[tt]);
      acc[tt] = fmaf(r.z, w2, acc[tt]);
      acc[tt] = fmaf(r.w, w3, acc[tt]);
    }
  }
  float* out = x + ((static_cast<long long>(c) * gridDim.y + band) * frames) * DIM + n;
#pragma unroll
  for (int tt = 0; tt < kBandFrames; ++tt)
    if (t0 + tt < frames) out[static_cast<long long>(t0 + tt) * DIM] = acc[tt];
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

// The same statistics for rows of DIM columns (one warp per row, DIM / 128
// float4 per lane), inv = sqrt(DIM) / sqrt(sum x^2 + 1e-12).
template <typename T, int DIM>
__global__ void __launch_bounds__(256) row_stats_dim_kernel(const float* __restrict__ x, long long rows,
                                                            T* __restrict__ x16, float* __restrict__ inv) {
  constexpr int kPer = DIM / 128;
  const long long r = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int lane = threadIdx.x & 31;
  const float4* src = reinterpret_cast<const float4*>(x + r * DIM);
  float4 a[kPer];
#pragma unroll
  for (int i = 0; i < kPer; ++i) a[i] = src[32 * i + lane];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) ss += a[i].x * a[i].x + a[i].y * a[i].y + a[i].z * a[i].z + a[i].w * a[i].w;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  T* dst = x16 + r * DIM;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    uint2 p;
    p.x = ElemTraits<T>::pack2(a[i].x, a[i].y);
    p.y = ElemTraits<T>::pack2(a[i].z, a[i].w);
    *reinterpret_cast<uint2*>(dst + 128 * i + lane * 4) = p;
  }
  if (lane == 0) inv[r] = sqrtf(static_cast<float>(DIM)) / sqrtf(ss + 1.0e-12f);
}

// Row factor from the sums of squares that the column tiles of a residual GEMM
// accumulated, and the sums cleared for the next residual GEMM.
__global__ void __launch_bounds__(256) norm_finalize_kernel(float* __restrict__ sumsq, float* __restrict__ inv,
                                                            long long rows, float scale) {
  const long long r = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  inv[r] = scale / sqrtf(sumsq[r] + 1.0e-12f);
  sumsq[r] = 0.f;
}

// ---------------------------------------------------------------- iSTFT
// Inverse of the STFT frame transform, one warp per (frame, channel), four
// frames per CTA.  Y = spec * mask (complex); the 2048-point inverse real FFT is
// a 1024-point complex FFT of Z[k] = (Y[k] + conj Y[1024-k]) +
// i e^{+2 pi i k / 2048} (Y[k] - conj Y[1024-k]): lane n2 gathers conj(Z) at
// k = 32 n1 + n2, the four-step forward FFT of stft_kernel runs, and the
// conjugate of the result, / 2048 and windowed, is the frame:
// x[2m] + i x[2m+1] = conj(FFT(conj Z))[m] / 2048.  The imaginary parts of
// Y[0] and Y[1024] do not reach the real inverse and are dropped.
__global__ void __launch_bounds__(256, 3) istft_frames_kernel(const float* __restrict__ spec,
                                                              const float* __restrict__ mask, int frames,
                                                              const float* __restrict__ window,
                                                              const float2* __restrict__ twiddle,
                                                              float* __restrict__ frames_out) {
  extern __shared__ float2 stft_smem[];
  float2* tw = stft_smem;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float2* buf = stft_smem + kStftTw + warp * kStftBuf;
  for (int k = threadIdx.x; k < 1025; k += blockDim.x) tw[k] = twiddle[k];
  const int f = blockIdx.x * kStftFramesPerCta + (warp >> 1);
  const int ch = warp & 1;
  const int c = blockIdx.y;
  const bool active = f < frames;   // warp-uniform
  const long long base = ((static_cast<long long>(c) * frames + (active ? f : 0)) * kFreqBins) * 4 + 2 * ch;
  auto bin = [&](int k) {   // Y[k] of this channel
    const float2 sv = *reinterpret_cast<const float2*>(spec + base + 4ll * k);
    const float2 mv = *reinterpret_cast<const float2*>(mask + base + 4ll * k);
    float2 y = make_float2(sv.x * mv.x - sv.y * mv.y, sv.x * mv.y + sv.y * mv.x);
    if (k == 0 || k == 1024) y.y = 0.f;
    return y;
  };
  float2 a[32];
#pragma unroll
  for (int n1 = 0; n1 < 32; ++n1) {
    const int k = 32 * n1 + lane;
    a[n1] = make_float2(0.f, 0.f);
    if (active) {
      const float2 ya = bin(k), yb = bin(1024 - k);
      const float2 t = __ldg(twiddle + k);
      const float2 e = make_float2(t.x, -t.y);
      const float2 sum = make_float2(ya.x + yb.x, ya.y - yb.y);
      const float2 dif = make_float2(ya.x - yb.x, ya.y + yb.y);
      const float2 ed = cmul(e, dif);
      a[n1] = make_float2(sum.x - ed.y, -(sum.y + ed.x));   // conj(Z[k])
    }
  }
  __syncthreads();   // twiddle table in shared memory ready
  if (!active) return;
  fft32(a, tw);
#pragma unroll
  for (int k1 = 1; k1 < 32; ++k1) a[k1] = cmul(a[k1], tw2048(tw, 2 * ((lane * k1) & 1023)));
#pragma unroll
  for (int k1 = 0; k1 < 32; ++k1) buf[k1 * 33 + lane] = a[k1];
  __syncwarp();
#pragma unroll
  for (int n2 = 0; n2 < 32; ++n2) a[n2] = buf[lane * 33 + n2];
  fft32(a, tw);   // a[k2] = FFT(conj Z)[lane + 32 k2]
  const float scale = 1.0f / 2048.0f;
  float2* dst = reinterpret_cast<float2*>(frames_out + ((static_cast<long long>(c) * 2 + ch) * frames + f) * kNfft);
#pragma unroll
  for (int k2 = 0; k2 < 32; ++k2) {
    const int m = lane + 32 * k2;
    const float2 w = *reinterpret_cast<const float2*>(window + 2 * m);
    dst[m] = make_float2(a[k2].x * scale * w.x, -a[k2].y * scale * w.y);
  }
}

__global__ void __launch_bounds__(256) overlap_add_kernel(const float* __restrict__ frames_buf, int frames,
                                                          int seg_length, int hop, const float* __restrict__ window,
                                                          float* __restrict__ seg_out) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= seg_length) return;
  const int cc = blockIdx.y;  // segment * 2 + channel
  // Frames f with f*hop - 1024 <= s < f*hop + 1024, i.e. f in
  // [q - ceil(2048 / hop) + 1, q] with q = floor((s + 1024) / hop) (s >= 0, so
  // the division is a floor); [q - 3, q] for hop 512.
  const int q = (s + kNfft / 2) / hop;
  const int f_hi = min(frames - 1, q);
  const int f_lo = max(0, q - ((kNfft + hop - 1) / hop - 1));
  float acc = 0.f, env = 0.f;
  const float* fb = frames_buf + static_cast<long long>(cc) * frames * kNfft;
  for (int f = f_lo; f <= f_hi; ++f) {
    const int i = s - (f * hop - kNfft / 2);
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
                        const float2* twiddle, float* spec, cudaStream_t stream, int hop) {
  if (segments <= 0 || frames <= 0) return cudaSuccess;
  if (hop <= 0 || hop > kNfft) return cudaErrorInvalidValue;
  static std::atomic<unsigned long long> configured{0};
  const cudaError_t e = opt_in_smem(stft_kernel, kStftSmem, configured);
  if (e != cudaSuccess) return e;
  stft_kernel<<<dim3((frames + kStftFramesPerCta - 1) / kStftFramesPerCta, segments), 256, kStftSmem, stream>>>(
      audio, map, frames, hop, window, twiddle, spec);
  return cudaGetLastError();
}

cudaError_t launch_band_split(const float* spec, int segments, int frames, const float* band_wt,
                              const long long* band_wt_offset, const float* band_gamma, const int* band_gamma_offset,
                              const float* band_bias, float* x, cudaStream_t stream, int dim, int bands) {
  static std::atomic<unsigned long long> configured256{0}, configured512{0};
  const int smem = kBandFrames * 516 * 4;   // widest band: 129 bins x 2 channels x re/im
  if (segments <= 0 || frames <= 0 || bands <= 0) return cudaSuccess;
  dim3 grid((frames + kBandFrames - 1) / kBandFrames, bands, segments);
  if (dim == 256) {
    const cudaError_t e = opt_in_smem(band_split_kernel<256>, smem, configured256);
    if (e != cudaSuccess) return e;
    band_split_kernel<256><<<grid, 256, smem, stream>>>(spec, frames, band_wt, band_wt_offset, band_gamma,
                                                         band_gamma_offset, band_bias, x);
  } else if (dim == 512) {
    const cudaError_t e = opt_in_smem(band_split_kernel<512>, smem, configured512);
    if (e != cudaSuccess) return e;
    band_split_kernel<512><<<grid, 512, smem, stream>>>(spec, frames, band_wt, band_wt_offset, band_gamma,
                                                         band_gamma_offset, band_bias, x);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_row_stats_dim(const float* x, long long rows, int dim, void* x16, float* inv, bool bf16,
                                 cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const unsigned blocks = static_cast<unsigned>((rows + 7) / 8);
  if (dim == 256) {
    if (bf16)
      row_stats_dim_kernel<__nv_bfloat16, 256><<<blocks, 256, 0, stream>>>(x, rows, static_cast<__nv_bfloat16*>(x16), inv);
    else
      row_stats_dim_kernel<__half, 256><<<blocks, 256, 0, stream>>>(x, rows, static_cast<__half*>(x16), inv);
  } else if (dim == 512) {
    if (bf16)
      row_stats_dim_kernel<__nv_bfloat16, 512><<<blocks, 256, 0, stream>>>(x, rows, static_cast<__nv_bfloat16*>(x16), inv);
    else
      row_stats_dim_kernel<__half, 512><<<blocks, 256, 0, stream>>>(x, rows, static_cast<__half*>(x16), inv);
  } else {
    return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_norm_finalize(float* sumsq, float* inv, long long rows, float scale, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  norm_finalize_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(sumsq, inv, rows, scale);
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
  static std::atomic<unsigned long long> configured{0};
  const cudaError_t e = opt_in_smem(istft_frames_kernel, kStftSmem, configured);
  if (e != cudaSuccess) return e;
  istft_frames_kernel<<<dim3((frames + kStftFramesPerCta - 1) / kStftFramesPerCta, segments), 256, kStftSmem,
                        stream>>>(spec, mask, frames, window, twiddle, frames_out);
  return cudaGetLastError();
}

cudaError_t launch_overlap_add(const float* frames_buf, int segments, int frames, int seg_length, const float* window,
                               float* seg_out, cudaStream_t stream, int hop) {
  if (segments <= 0 || seg_length <= 0) return cudaSuccess;
  if (hop <= 0 || hop > kNfft) return cudaErrorInvalidValue;
  dim3 grid((seg_length + 255) / 256, segments * 2);
  overlap_add_kernel<<<grid, 256, 0, stream>>>(frames_buf, frames, seg_length, hop, window, seg_out);
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
