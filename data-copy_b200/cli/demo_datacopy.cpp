// demo_datacopy: runs one standalone_datacopy mode on a B200 through the dcopy C ABI
// and checks the transpose on the host.
//
//   demo_datacopy small|large|pretranspose ROWS COLS TILE_KIB STORE(0|1) DEVICE_ID
//                 [VERIFICATION_FILE]
//
// The command line, the error texts, the input pattern (word i holds i*17+3),
// the 0xA5 canary in y and the one-line report file follow the reference's
// host program (standalone_datacopy/datacopy_data_collection.asc:97-181), so
// scripts written for it (profile.py) drive this tool unchanged.  The tiling
// itself is validated by dcopy_plan_tiling, whose messages are the reference's.
// The summary line keeps the reference's keys and adds the device time of the
// timed launch (CUDA events) and the GB/s it moved.
#include <cuda_runtime.h>

#include <algorithm>
#include <cctype>
#include <cstdint>
#include <cstdlib>
#include <fstream>
#include <iostream>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "dcopy/dcopy.h"

namespace {

struct Failure : std::runtime_error {
  using std::runtime_error::runtime_error;
};

void cuda_ok(cudaError_t e, const char *what) {
  if (e != cudaSuccess) throw Failure(std::string(what) + ": " + cudaGetErrorName(e));
}
void dcopy_ok(int rc) {
  if (rc != DCOPY_OK) throw Failure(dcopy_last_error_message());
}

// ---- command line ----------------------------------------------------------------

enum class Mode { kSmall, kLarge, kPretranspose };

struct Options {
  Mode mode;
  std::string mode_name;
  uint32_t rows, cols, tile_kib, store, device;
  const char *report = nullptr;  // VERIFICATION_FILE, only with STORE=1
};

// A decimal u32: digits only (no sign, no blank), at most 4294967295.
uint32_t parse_u32(const std::string &text) {
  const bool digits = !text.empty() && std::all_of(text.begin(), text.end(), [](unsigned char ch) {
    return std::isdigit(ch) != 0;
  });
  if (!digits) throw Failure("Expected a nonnegative integer");
  uint64_t v = 0;
  for (char ch : text) {
    v = v * 10 + uint64_t(ch - '0');
    if (v > 0xFFFFFFFFull) throw Failure("Integer overflow");
  }
  return uint32_t(v);
}

Options parse(int argc, char **argv) {
  if (argc < 7 || argc > 8)
    throw Failure(
        "Usage: demo_datacopy small|large|pretranspose ROWS COLS TILE_KIB STORE(0|1) DEVICE_ID "
        "[VERIFICATION_FILE]");
  static const std::pair<const char *, Mode> kModes[] = {
      {"small", Mode::kSmall}, {"large", Mode::kLarge}, {"pretranspose", Mode::kPretranspose}};
  Options o{};
  o.mode_name = argv[1];
  const auto *hit = std::find_if(std::begin(kModes), std::end(kModes),
                                 [&](const auto &m) { return o.mode_name == m.first; });
  if (hit == std::end(kModes)) throw Failure("Unknown mode");
  o.mode = hit->second;
  uint32_t *fields[] = {&o.rows, &o.cols, &o.tile_kib, &o.store, &o.device};
  for (int i = 0; i < 5; ++i) *fields[i] = parse_u32(argv[2 + i]);
  if (argc == 8) {
    if (o.store != 1) throw Failure("VERIFICATION_FILE requires STORE=1");
    o.report = argv[7];
  }
  return o;
}

// ---- device buffers -------------------------------------------------------------

// Owns the run's stream and device buffers.  The destructor drains the stream
// before anything is freed, on success and on every error path alike.
class Session {
 public:
  explicit Session(int device) {
    cuda_ok(cudaSetDevice(device), "cudaSetDevice");
    cuda_ok(cudaStreamCreate(&stream_), "cudaStreamCreate");
  }
  ~Session() {
    cudaStreamSynchronize(stream_);
    for (void *p : owned_) cudaFree(p);
    cudaStreamDestroy(stream_);
  }
  Session(const Session &) = delete;
  Session &operator=(const Session &) = delete;

  void *alloc(size_t bytes) {
    void *p = nullptr;
    cuda_ok(cudaMalloc(&p, bytes), "cudaMalloc");
    owned_.push_back(p);
    return p;
  }
  cudaStream_t stream() const { return stream_; }
  dcopy_stream_t handle() const { return reinterpret_cast<dcopy_stream_t>(stream_); }

 private:
  cudaStream_t stream_ = nullptr;
  std::vector<void *> owned_;
};

// ---- the run ----------------------------------------------------------------------

// The mode's kernels in stream order: pretranspose writes B, then copies B to y.
void launch_mode(Mode mode, const void *x, void *y, void *b, const DataCopyTiling *t,
                 dcopy_stream_t s) {
  switch (mode) {
    case Mode::kSmall: dcopy_ok(dcopy_datacopy_small(x, y, t, s)); break;
    case Mode::kLarge: dcopy_ok(dcopy_datacopy_large(x, y, t, s)); break;
    case Mode::kPretranspose:
      dcopy_ok(dcopy_datacopy_pretranspose(x, b, t, s));
      dcopy_ok(dcopy_datacopy_contiguous(b, y, t, s));
      break;
  }
}

std::string run(const Options &o) {
  DataCopyTiling tiling{};
  dcopy_ok(dcopy_plan_tiling(o.rows, o.cols, o.tile_kib, o.store, &tiling));
  if (o.device > 255) throw Failure("device: 0..255");
  const size_t words = size_t(tiling.rows) * tiling.cols, bytes = words * 4;
  // Word i of the input is i*17+3 (wrapping in 32 bits), as the reference fills it.
  std::vector<uint32_t> host(words);
  for (size_t i = 0; i < words; ++i) host[i] = uint32_t(i) * 17u + 3u;

  Session dev(int(o.device));
  const bool two_pass = o.mode == Mode::kPretranspose;
  void *x = dev.alloc(bytes), *y = dev.alloc(bytes), *b = dev.alloc(two_pass ? bytes : 16);
  auto *tiling_dev = static_cast<DataCopyTiling *>(dev.alloc(sizeof(tiling)));
  cuda_ok(cudaMemcpy(x, host.data(), bytes, cudaMemcpyHostToDevice), "input upload");
  cuda_ok(cudaMemcpy(tiling_dev, &tiling, sizeof(tiling), cudaMemcpyHostToDevice), "tiling upload");

  // First launch with the tiling in device memory, as the reference hands it to
  // its kernels; it also loads the kernels' module, so the timed launch below
  // (host tiling: no synchronising read) measures the copy alone.
  launch_mode(o.mode, x, y, b, tiling_dev, dev.handle());
  if (tiling.store) cuda_ok(cudaMemsetAsync(y, 0xA5, bytes, dev.stream()), "canary");
  cudaEvent_t ev[2];
  for (cudaEvent_t &e : ev) cuda_ok(cudaEventCreate(&e), "cudaEventCreate");
  cuda_ok(cudaEventRecord(ev[0], dev.stream()), "cudaEventRecord");
  launch_mode(o.mode, x, y, b, &tiling, dev.handle());
  cuda_ok(cudaEventRecord(ev[1], dev.stream()), "cudaEventRecord");
  cuda_ok(cudaStreamSynchronize(dev.stream()), "cudaStreamSynchronize");
  float ms = 0.f;
  cuda_ok(cudaEventElapsedTime(&ms, ev[0], ev[1]), "cudaEventElapsedTime");
  for (cudaEvent_t e : ev) cudaEventDestroy(e);

  if (tiling.store) {
    // y = x transposed: y word (c, r) must hold the input value of word r*cols + c.
    cuda_ok(cudaMemcpy(host.data(), y, bytes, cudaMemcpyDeviceToHost), "result download");
    for (size_t j = 0; j < words; ++j) {
      const size_t c = j / tiling.rows, r = j % tiling.rows;
      if (host[j] != uint32_t(r * tiling.cols + c) * 17u + 3u)
        throw Failure("Transpose verification failed at " + std::to_string(r) + "," +
                      std::to_string(c));
    }
  }
  // Device bytes per launch sequence: x read, plus y (and B) written when stored.
  const double moved = double(bytes) * (two_pass ? 4.0 : (tiling.store ? 2.0 : 1.0));
  std::ostringstream line;
  line << "mode=" << o.mode_name << " rows=" << tiling.rows << " cols=" << tiling.cols
       << " input_bytes=" << bytes << " tile_cols=" << tiling.tile_cols
       << " tile_count=" << (tiling.cols + tiling.tile_cols - 1) / tiling.tile_cols
       << " ub_bytes=" << tiling.ub_bytes
       << " verification=" << (tiling.store ? "PASS" : "not_requested")
       << " kernel_us=" << ms * 1e3 << " gbps=" << moved / (double(ms) * 1e6);
  return line.str();
}

}  // namespace

int main(int argc, char **argv) {
  Options opts{};
  try {
    opts = parse(argc, argv);
    std::cout << run(opts) << '\n';  // every device resource is released by now
  } catch (const std::exception &e) {
    std::cerr << e.what() << '\n';
    return 1;
  }
  if (opts.report) {  // written only once the run and its cleanup have succeeded
    std::ofstream out(opts.report);
    out << "verification=PASS\n";
    if (!out.flush()) {
      std::cerr << "Cannot write verification report: " << opts.report << '\n';
      return 1;
    }
  }
  return 0;
}
