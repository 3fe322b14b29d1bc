// Batch separation of WAV files with the file I/O off the critical path.
//
// vocalarc_b200_separate_files keeps three stages busy at once: a reader
// thread decodes track i+1, the calling thread separates track i on the
// device, and a writer thread writes track i-1.  Two-slot queues between the
// stages bound the memory to a few tracks.  The file formats and conversions
// are the reference host's (native/vocalarc_separation.c):
//   * wav_read :1152-1187 -- RIFF/WAVE, PCM 16/24/32-bit or float32, mono or
//     stereo, any rate; the last "fmt " and "data" chunks win; samples to
//     planar float32;
//   * to_stereo :1189-1196 -- mono is duplicated;
//   * resample_linear :1198-1222 -- to 44.1 kHz, align_corners=False linear
//     interpolation, length llround(n * 44100 / rate);
//   * wav_write :1224-1237 -- 44-byte float32 stereo 44.1 kHz header,
//     non-finite samples written as 0; instrumental = mix - vocals (:1587-1593).
// Host code only; the device work is vocalarc_b200_separate(_chunked).
#include <cmath>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "vocalarc_b200.h"

namespace {

constexpr int kRate = 44100;

uint16_t le16(const unsigned char* p) { return static_cast<uint16_t>(p[0] | (p[1] << 8)); }
uint32_t le32(const unsigned char* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
         (static_cast<uint32_t>(p[3]) << 24);
}
void put16(unsigned char* p, uint16_t v) {
  p[0] = static_cast<unsigned char>(v);
  p[1] = static_cast<unsigned char>(v >> 8);
}
void put32(unsigned char* p, uint32_t v) {
  for (int i = 0; i < 4; ++i) p[i] = static_cast<unsigned char>(v >> (8 * i));
}

bool read_bytes(const char* path, std::vector<unsigned char>& out) {
  FILE* f = fopen(path, "rb");
  if (f == nullptr) return false;
  bool ok = fseek(f, 0, SEEK_END) == 0;
  const long size = ok ? ftell(f) : -1;
  ok = ok && size >= 0 && fseek(f, 0, SEEK_SET) == 0;
  if (ok) {
    out.resize(static_cast<size_t>(size));
    ok = size == 0 || fread(out.data(), 1, out.size(), f) == out.size();
  }
  fclose(f);
  return ok;
}

// Decoded track: planar stereo float32 at 44.1 kHz.
bool read_track(const char* path, std::vector<float>& stereo, int& length) {
  std::vector<unsigned char> file;
  if (!read_bytes(path, file) || file.size() < 44 || memcmp(file.data(), "RIFF", 4) != 0 ||
      memcmp(file.data() + 8, "WAVE", 4) != 0) {
    fprintf(stderr, "vocalarc-b200: unsupported WAV input: %s\n", path);
    return false;
  }
  const size_t size = file.size();
  int format = 0, channels = 0, rate = 0, bits = 0;
  const unsigned char* data = nullptr;
  uint32_t data_size = 0;
  size_t offset = 12;
  while (offset + 8 <= size) {
    const unsigned char* chunk = file.data() + offset;
    const uint32_t chunk_size = le32(chunk + 4);
    const size_t payload = offset + 8;
    if (payload > size || chunk_size > size - payload) break;
    if (memcmp(chunk, "fmt ", 4) == 0 && chunk_size >= 16) {
      format = le16(file.data() + payload);
      channels = le16(file.data() + payload + 2);
      rate = static_cast<int>(le32(file.data() + payload + 4));
      bits = le16(file.data() + payload + 14);
    } else if (memcmp(chunk, "data", 4) == 0) {
      data = file.data() + payload;
      data_size = chunk_size;
    }
    offset = payload + chunk_size + (chunk_size & 1u);
  }
  if (data == nullptr || channels < 1 || channels > 2 || rate < 1 || (format != 1 && format != 3) ||
      (format == 1 && bits != 16 && bits != 24 && bits != 32) || (format == 3 && bits != 32)) {
    fprintf(stderr, "vocalarc-b200: WAV must be PCM16/24/32 or float32 mono/stereo: %s\n", path);
    return false;
  }
  const int bytes = bits / 8;
  const size_t frame_bytes = static_cast<size_t>(channels) * bytes;
  const int n = static_cast<int>(data_size / frame_bytes);
  std::vector<float> planar(static_cast<size_t>(channels) * n);
  for (int i = 0; i < n; ++i)
    for (int c = 0; c < channels; ++c) {
      const unsigned char* p = data + static_cast<size_t>(i) * frame_bytes + static_cast<size_t>(c) * bytes;
      float value;
      if (format == 3) {
        memcpy(&value, p, sizeof(value));
      } else if (bits == 16) {
        value = static_cast<float>(static_cast<int16_t>(le16(p))) / 32768.0f;
      } else if (bits == 24) {
        int32_t v = static_cast<int32_t>(p[0]) | (static_cast<int32_t>(p[1]) << 8) | (static_cast<int32_t>(p[2]) << 16);
        if (v & 0x800000) v |= ~0xffffff;
        value = static_cast<float>(v) / 8388608.0f;
      } else {
        value = static_cast<float>(static_cast<int32_t>(le32(p))) / 2147483648.0f;
      }
      planar[static_cast<size_t>(c) * n + i] = value;
    }
  // Mono -> stereo by duplication.
  std::vector<float> two(2 * static_cast<size_t>(n));
  memcpy(two.data(), planar.data(), static_cast<size_t>(n) * sizeof(float));
  memcpy(two.data() + n, planar.data() + (channels == 2 ? n : 0), static_cast<size_t>(n) * sizeof(float));
  if (rate == kRate) {
    stereo.swap(two);
    length = n;
    return true;
  }
  // Linear resampling to 44.1 kHz (align_corners=False).
  int out_len = static_cast<int>(llround(static_cast<double>(n) * kRate / rate));
  if (out_len < 1) out_len = 1;
  if (n < 1) {
    fprintf(stderr, "vocalarc-b200: empty WAV input: %s\n", path);
    return false;
  }
  stereo.assign(2 * static_cast<size_t>(out_len), 0.0f);
  for (int c = 0; c < 2; ++c) {
    const float* src = two.data() + static_cast<size_t>(c) * n;
    float* dst = stereo.data() + static_cast<size_t>(c) * out_len;
    for (int i = 0; i < out_len; ++i) {
      double position = (static_cast<double>(i) + 0.5) * rate / kRate - 0.5;
      if (position < 0.0) position = 0.0;
      double upper_position = position + 1.0;
      if (upper_position > n - 1) upper_position = n - 1;
      const int lower = static_cast<int>(position);
      const int upper = static_cast<int>(upper_position);
      const float fraction = static_cast<float>(position - lower);
      dst[i] = src[lower] * (1.0f - fraction) + src[upper] * fraction;
    }
  }
  length = out_len;
  return true;
}

bool write_track(const char* path, const float* planar, int length) {
  FILE* f = fopen(path, "wb");
  if (f == nullptr) return false;
  const uint32_t data_size = static_cast<uint32_t>(static_cast<size_t>(length) * 2 * sizeof(float));
  unsigned char header[44] = {0};
  memcpy(header, "RIFF", 4);
  put32(header + 4, 36 + data_size);
  memcpy(header + 8, "WAVEfmt ", 8);
  put32(header + 16, 16);
  put16(header + 20, 3);
  put16(header + 22, 2);
  put32(header + 24, kRate);
  put32(header + 28, kRate * 2 * sizeof(float));
  put16(header + 32, 2 * sizeof(float));
  put16(header + 34, 32);
  memcpy(header + 36, "data", 4);
  put32(header + 40, data_size);
  bool ok = fwrite(header, 1, sizeof(header), f) == sizeof(header);
  std::vector<float> frames(2 * static_cast<size_t>(length));
  for (int i = 0; i < length; ++i)
    for (int c = 0; c < 2; ++c) {
      const float v = planar[static_cast<size_t>(c) * length + i];
      frames[2 * static_cast<size_t>(i) + c] = std::isfinite(v) ? v : 0.0f;
    }
  ok = ok && (frames.empty() || fwrite(frames.data(), sizeof(float), frames.size(), f) == frames.size());
  return fclose(f) == 0 && ok;
}

struct Track {
  int index = -1;
  int length = 0;
  bool ok = false;
  std::vector<float> mix;
  std::vector<float> vocals;
};

// Bounded single-producer / single-consumer queue; pop returns false once the
// queue is closed and drained.
class Channel {
 public:
  explicit Channel(size_t depth) : depth_(depth) {}
  void push(Track&& t) {
    std::unique_lock<std::mutex> lock(m_);
    not_full_.wait(lock, [&] { return q_.size() < depth_; });
    q_.push_back(std::move(t));
    not_empty_.notify_one();
  }
  bool pop(Track& t) {
    std::unique_lock<std::mutex> lock(m_);
    not_empty_.wait(lock, [&] { return !q_.empty() || closed_; });
    if (q_.empty()) return false;
    t = std::move(q_.front());
    q_.pop_front();
    not_full_.notify_one();
    return true;
  }
  void close() {
    std::lock_guard<std::mutex> lock(m_);
    closed_ = true;
    not_empty_.notify_all();
  }

 private:
  size_t depth_;
  bool closed_ = false;
  std::deque<Track> q_;
  std::mutex m_;
  std::condition_variable not_full_, not_empty_;
};

}  // namespace

extern "C" int vocalarc_b200_read_track(const char* path, float* out, long long capacity, int* length) {
  if (path == nullptr || length == nullptr) return 0;
  std::vector<float> stereo;
  int n = 0;
  if (!read_track(path, stereo, n)) return 0;
  *length = n;
  if (out == nullptr) return 1;
  if (capacity < 2ll * n) return 0;
  memcpy(out, stereo.data(), stereo.size() * sizeof(float));
  return 1;
}

extern "C" int vocalarc_b200_write_track(const char* path, const float* audio, int length) {
  if (path == nullptr || audio == nullptr || length < 0) return 0;
  return write_track(path, audio, length) ? 1 : 0;
}

extern "C" int vocalarc_b200_separate_files(native_gpu* gpu, int count, const char* const* input_paths,
                                            const char* const* vocals_paths, const char* const* instrumental_paths,
                                            int chunked) {
  if (gpu == nullptr || count <= 0 || input_paths == nullptr || vocals_paths == nullptr) return 0;
  Channel decoded(2), separated(2);
  std::thread reader([&] {
    for (int i = 0; i < count; ++i) {
      Track t;
      t.index = i;
      t.ok = input_paths[i] != nullptr && read_track(input_paths[i], t.mix, t.length);
      decoded.push(std::move(t));
    }
    decoded.close();
  });
  int written = 0;
  std::thread writer([&] {
    Track t;
    while (separated.pop(t)) {
      if (!t.ok) continue;
      bool ok = vocals_paths[t.index] != nullptr && write_track(vocals_paths[t.index], t.vocals.data(), t.length);
      const char* inst = instrumental_paths != nullptr ? instrumental_paths[t.index] : nullptr;
      if (ok && inst != nullptr && inst[0] != '\0') {
        for (size_t k = 0; k < t.mix.size(); ++k) t.mix[k] -= t.vocals[k];
        ok = write_track(inst, t.mix.data(), t.length);
      }
      if (ok)
        ++written;
      else
        fprintf(stderr, "vocalarc-b200: cannot write the outputs of track %d\n", t.index);
    }
  });
  Track t;
  while (decoded.pop(t)) {
    if (t.ok) {
      t.vocals.assign(t.mix.size(), 0.0f);
      t.ok = chunked ? vocalarc_b200_separate_chunked(gpu, t.mix.data(), t.length, 0, 1, t.vocals.data()) != 0
                     : vocalarc_b200_separate(gpu, t.mix.data(), t.length, t.vocals.data()) != 0;
      if (!t.ok) fprintf(stderr, "vocalarc-b200: separation of track %d failed\n", t.index);
    }
    separated.push(std::move(t));
  }
  separated.close();
  reader.join();
  writer.join();
  return written;
}
