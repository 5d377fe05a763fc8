// dcopy_bench: the C++ measurement tool of the library (it replaces the reference's
// msprof harness standalone_datacopy/profile.py and its host address model
// test_address_model.py).  Every result is verified on the host before it is timed.
//
//   dcopy_bench sweep [--moved-mib M] [--blens L,...] [--gaps G,...] [--reps R] [--device D]
//       blockLen x gap sweep (gaps as multiples of blockLen) of dcopy_copy_ext on an int32
//       element-index source; one JSON line per point with measured GB/s, the
//       fraction of the copy peak and a DRAM-atom model of the achievable rate.
//   dcopy_bench standalone ROWS COLS SMALL_KIB LARGE_KIB [--trials N] [--device D]
//                          [--output DIR] [--peak GBPS]
//       profile.py main(): verify small/large/pretranspose with STORE=1, then time
//       `trials` rounds with STORE=0 in rotated order and write config.json,
//       raw.csv, stages.csv and summary.json (device time per kernel from CUDA
//       events in place of msprof's Task Duration).
//   dcopy_bench nz [--batch B] [--h H] [--w W] [--c0 C] [--format nz|zz] [--reps R]
//                  [--device D]
//       fp16 ND -> FRACTAL_NZ -> ND (or FRACTAL_ZZ), round trip
//       verified.
//   dcopy_bench pcie [--rows R] [--len L] [--pitch P] [--reps N] [--device D]
//       The copy engine over PCIe as the staged host-to-host copy uses it: 2-D
//       gathers host -> device, contiguous copies each way, each cut into 1, 4,
//       16 and 64 copies, and both directions at once; one JSON line per case.
//   dcopy_bench staged [--calls C] [--reps R] [--device D]
//       BASELINE config 2 end to end from pinned host memory through
//       dcopy_copy_ext_staged: device time and host issue time per call, verified.
//   dcopy_bench fz [--n N] [--c C] [--h H] [--w W] [--eb B] [--c0 C0] [--reps R]
//                  [--replay 0|1] [--formats nchw,nhwc,hwcn] [--device D] [--peak GBPS]
//       Convolution weights: NCHW / NHWC / HWCN -> FRACTAL_Z -> back, each
//       round trip verified; one JSON line per format.  --replay 1 times graph
//       replays of two alternating weight sets without L2 eviction.
//   dcopy_bench transpose --shape A,B,C,D --perm P0,P1,P2,P3 [--eb B] [--reps R]
//                         [--device D] [--peak GBPS]
//       GE Transpose (dcopy_transpose) of a dense tensor, verified against a host
//       restatement; one JSON line.
//   dcopy_bench nd [--sizes A,B,C[,D,E]] [--eb B] [--src-pad P] [--dst-pad Q] [--tma 0|1]
//                  [--src-order O0,O1,..] [--dst-order O0,O1,..] [--reps R] [--device D]
//                  [--peak GBPS]
//       DataCopyNddma box (dcopy_copy_nd) between padded views, verified; one JSON
//       line: event time around the call, the same call replayed as a CUDA graph,
//       and the host time of one call.  --tma 1 selects the TMA tensor-copy path
//       (dcopy_set_nd_tma) for boxes that qualify.
//   dcopy_bench batch [--gathers G] [--reps R] [--device D] [--peak GBPS]
//       G config-2 gathers as one dcopy_copy_ext_batch against G dcopy_copy_ext calls
//       (both captured in a CUDA graph), verified; one JSON line.
//   dcopy_bench p2p [--mib M | --kib K] [--reps R] [--device D] [--peer P] [--peak GBPS]
//       NVLink between two GPUs: dcopy_p2p_copy as a push launched on the
//       sending GPU (automatic engine choice, then the SM engine forced), as a
//       pull launched on the receiving GPU, cudaMemcpyPeerAsync, and the two
//       halves split SM push + copy engine or push + pull; each with both GPUs
//       sending at once and with one sending.
//
// Timing: 3 untimed warm-up calls, then CUDA events around each launch (median of
// 20 reps by default); a 512 MiB read between reps (load-only
// mode, so L2 holds only clean lines) evicts the 126 MB L2: every rep reads cold
// data and no flush write-back falls inside the timed region.
#include <cuda_runtime.h>
#include <sys/stat.h>

#include <algorithm>
#include <cctype>
#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <functional>
#include <iostream>
#include <map>
#include <memory>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "dcopy/dcopy.h"

namespace {

void Check(cudaError_t e, const char *what) {
  if (e != cudaSuccess)
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorName(e));
}

void CheckD(int rc) {
  if (rc != DCOPY_OK) throw std::runtime_error(dcopy_last_error_message());
}

struct Args {
  std::vector<std::string> pos;
  std::map<std::string, std::string> opt;
  Args(int argc, char **argv) {
    for (int i = 2; i < argc; ++i) {
      std::string a = argv[i];
      if (a.rfind("--", 0) == 0 && i + 1 < argc)
        opt[a.substr(2)] = argv[++i];
      else
        pos.push_back(a);
    }
  }
  double num(const std::string &k, double d) const {
    auto it = opt.find(k);
    return it == opt.end() ? d : std::stod(it->second);
  }
  bool has(const std::string &k) const { return opt.count(k) != 0; }
  std::string str(const std::string &k, const std::string &d) const {
    auto it = opt.find(k);
    return it == opt.end() ? d : it->second;
  }
};

struct DevBuf {
  void *p = nullptr;
  size_t n = 0;
  explicit DevBuf(size_t bytes) : n(bytes) { Check(cudaMalloc(&p, bytes), "cudaMalloc"); }
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  DevBuf(const DevBuf &) = delete;
  DevBuf &operator=(const DevBuf &) = delete;
};

// Evicts the measured buffers from L2 by reading `flush` (512 MiB) with the
// library's load-only mode: the lines left in L2 are clean, so no write-back of
// flush data lands inside the next timed region (a memset would leave ~126 MB of
// dirty lines to be written back while the measured kernel runs).
void read_flush(DevBuf &flush, cudaStream_t s) {
  DataCopyTiling t{};  // the flush buffer's contents are never used
  CheckD(dcopy_plan_tiling(4088, 4104, 240, 0, &t));  // 64 MiB of int32, load only
  const size_t chunk = size_t(4088) * 4104 * 4;
  for (size_t off = 0; off + chunk <= flush.n; off += size_t(64) << 20)
    CheckD(dcopy_datacopy_contiguous(static_cast<char *>(flush.p) + off, nullptr, &t,
                                     reinterpret_cast<dcopy_stream_t>(s)));
}

constexpr int kWarmupReps = 3;

// Times `fn` (one or more launches on `s`) `reps` times with an L2 flush between reps,
// after kWarmupReps untimed calls.
template <typename F>
std::vector<double> time_reps(F fn, int reps, cudaStream_t s, DevBuf &flush) {
  cudaEvent_t a, b;
  Check(cudaEventCreate(&a), "event");
  Check(cudaEventCreate(&b), "event");
  for (int r = 0; r < kWarmupReps; ++r) fn();  // untimed warm-up
  Check(cudaStreamSynchronize(s), "sync");
  std::vector<double> us;
  for (int r = 0; r < reps; ++r) {
    read_flush(flush, s);
    Check(cudaEventRecord(a, s), "record");
    fn();
    Check(cudaEventRecord(b, s), "record");
    Check(cudaEventSynchronize(b), "sync");
    float ms = 0;
    Check(cudaEventElapsedTime(&ms, a, b), "elapsed");
    us.push_back(ms * 1e3);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return us;
}

// The same, with `fn` captured once into a CUDA graph and the graph replayed
// between the events: device time without the host work of the call.
template <typename F>
std::vector<double> time_graph_reps(F fn, int reps, cudaStream_t s, DevBuf &flush) {
  cudaGraph_t graph;
  cudaGraphExec_t exec;
  Check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
  fn();
  Check(cudaStreamEndCapture(s, &graph), "end capture");
  Check(cudaGraphInstantiate(&exec, graph, 0), "instantiate");
  auto us = time_reps([&] { Check(cudaGraphLaunch(exec, s), "graph launch"); }, reps, s, flush);
  cudaGraphExecDestroy(exec);
  cudaGraphDestroy(graph);
  return us;
}

// Steady-state device time of `fn` (microseconds per call): `fn` captured once
// into a CUDA graph, replayed back to back `reps` times between two events with
// no eviction between replays, so the write-back of each replay's dirty L2
// lines falls inside the next one, as in a long sequence of calls.
template <typename F>
double replay_us(F fn, int reps, cudaStream_t s) {
  cudaGraph_t graph;
  cudaGraphExec_t exec;
  Check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
  fn();
  Check(cudaStreamEndCapture(s, &graph), "end capture");
  Check(cudaGraphInstantiate(&exec, graph, 0), "instantiate");
  for (int r = 0; r < 5; ++r) Check(cudaGraphLaunch(exec, s), "graph launch");
  cudaEvent_t a, b;
  Check(cudaEventCreate(&a), "event");
  Check(cudaEventCreate(&b), "event");
  Check(cudaEventRecord(a, s), "record");
  for (int r = 0; r < reps; ++r) Check(cudaGraphLaunch(exec, s), "graph launch");
  Check(cudaEventRecord(b, s), "record");
  Check(cudaEventSynchronize(b), "sync");
  float ms = 0;
  Check(cudaEventElapsedTime(&ms, a, b), "elapsed");
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  cudaGraphExecDestroy(exec);
  cudaGraphDestroy(graph);
  return double(ms) * 1e3 / reps;
}

// Host time of one call of `fn` (asynchronous launches; the stream drains after).
template <typename F>
double host_us_per_call(F fn, int reps, cudaStream_t s) {
  double total = 0;
  for (int r = 0; r < reps; ++r) {
    const auto t0 = std::chrono::steady_clock::now();
    fn();
    const auto t1 = std::chrono::steady_clock::now();
    total += std::chrono::duration<double, std::micro>(t1 - t0).count();
    Check(cudaStreamSynchronize(s), "sync");
  }
  return total / reps;
}

double median(std::vector<double> v) {
  std::sort(v.begin(), v.end());
  const size_t n = v.size();
  return n % 2 ? v[n / 2] : 0.5 * (v[n / 2 - 1] + v[n / 2]);
}

std::vector<int64_t> parse_list(const std::string &text);

// ---- sweep ---------------------------------------------------------------------

// DRAM-atom model: HBM moves 64-byte atoms, so a burst of blen bytes that starts
// on a 64-byte boundary costs ceil(blen/64)*64 bytes read unless its neighbour
// burst shares the atom (gap 0); writes to the packed destination are whole atoms.
double model_gbps(double peak, uint64_t blen, uint64_t gap) {
  const double read = gap == 0 ? double(blen) : std::ceil(blen / 64.0) * 64.0;
  return peak * (2.0 * blen) / (read + blen);
}

int run_sweep(const Args &a) {
  const uint64_t moved = uint64_t(a.num("moved-mib", 256)) << 20;
  const int reps = int(a.num("reps", 20));
  const double peak = a.num("peak", 6543.4);
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  const uint64_t src_bytes = moved * 17;  // gap 16x
  DevBuf src(src_bytes), dst(moved), flush(512ull << 20);
  {  // int32 element-index source
    std::vector<int32_t> host(src_bytes / 4);
    for (size_t i = 0; i < host.size(); ++i) host[i] = int32_t(i);
    Check(cudaMemcpy(src.p, host.data(), src_bytes, cudaMemcpyHostToDevice), "H2D");
  }
  std::vector<int32_t> out(moved / 4);
  for (int64_t blen_ : parse_list(a.str("blens", "32,64,128,512,4096,65536"))) {
    for (int64_t gx_ : parse_list(a.str("gaps", "0,1,4,16"))) {
      const uint64_t blen = uint64_t(blen_), gx = uint64_t(gx_);
      if (blen < 4 || blen % 4 || moved % blen || gx > 16)
        throw std::runtime_error("sweep: blens must divide the moved bytes, gaps 0..16");
      const uint64_t gap = gx * blen, count = moved / blen;
      DcopyExtParams p{uint32_t(count), uint32_t(blen), gap, 0};
      Check(cudaMemsetAsync(dst.p, 0xA5, moved, s), "memset");
      CheckD(dcopy_copy_ext(dst.p, src.p, &p, reinterpret_cast<dcopy_stream_t>(s)));
      Check(cudaMemcpy(out.data(), dst.p, moved, cudaMemcpyDeviceToHost), "D2H");
      // Address model (test_address_model.py:24): dst word j comes from block
      // j / (blen/4) at word offset j % (blen/4) of source byte block*(blen+gap).
      const uint64_t wpb = blen / 4, spb = (blen + gap) / 4;
      for (uint64_t j = 0; j < out.size(); ++j) {
        const int32_t expect = int32_t((j / wpb) * spb + j % wpb);
        if (out[j] != expect)
          throw std::runtime_error("sweep mismatch at blen " + std::to_string(blen) + " gap " +
                                   std::to_string(gap) + " word " + std::to_string(j));
      }
      auto us = time_reps(
          [&] { CheckD(dcopy_copy_ext(dst.p, src.p, &p, reinterpret_cast<dcopy_stream_t>(s))); },
          reps, s, flush);
      const double med = median(us), gbps = 2.0 * moved / (med * 1e3);
      std::cout << "{\"config\": 3, \"blockLen\": " << blen << ", \"gap\": " << gap
                << ", \"blockCount\": " << count << ", \"moved_bytes\": " << moved
                << ", \"median_us\": " << med << ", \"GBps\": " << gbps
                << ", \"frac_of_peak\": " << gbps / peak
                << ", \"model_GBps\": " << model_gbps(peak, blen, gap)
                << ", \"frac_of_model\": " << gbps / model_gbps(peak, blen, gap)
                << ", \"verified\": true}" << std::endl;
    }
  }
  cudaStreamDestroy(s);
  return 0;
}

// ---- standalone (profile.py) ------------------------------------------------------

struct Stage {
  std::string kernel;
  double us;
};

int run_standalone(const Args &a) {
  if (a.pos.size() != 4)
    throw std::runtime_error("standalone ROWS COLS SMALL_KIB LARGE_KIB [--trials N] ...");
  const uint32_t rows = std::stoul(a.pos[0]), cols = std::stoul(a.pos[1]);
  const uint32_t small_kib = std::stoul(a.pos[2]), large_kib = std::stoul(a.pos[3]);
  const int trials = int(a.num("trials", 3));
  const int device = int(a.num("device", 0));
  const std::string outdir = a.str("output", "");
  if (trials < 1 || device < 0 || device > 255)
    throw std::runtime_error("trials >= 1; device: 0..255");
  DataCopyTiling small{}, large{};
  CheckD(dcopy_plan_tiling(rows, cols, small_kib, 1, &small));  // profile.py:133-137
  CheckD(dcopy_plan_tiling(rows, cols, large_kib, 1, &large));
  if (small.ub_bytes >= large.ub_bytes)
    throw std::runtime_error("Actual small tile must be smaller than large tile");
  if (!outdir.empty() && mkdir(outdir.c_str(), 0755) != 0)  // profile.py:158 exist_ok=False
    throw std::runtime_error("output directory must not exist: " + outdir);
  Check(cudaSetDevice(device), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  dcopy_stream_t ds = reinterpret_cast<dcopy_stream_t>(s);
  const size_t bytes = size_t(rows) * cols * 4;
  DevBuf x(bytes), y(bytes), b(bytes), flush(512ull << 20);
  std::vector<int32_t> input(bytes / 4), output(bytes / 4);
  for (size_t i = 0; i < input.size(); ++i) input[i] = int32_t(i * 17 + 3);
  Check(cudaMemcpy(x.p, input.data(), bytes, cudaMemcpyHostToDevice), "H2D");
  const std::vector<std::string> modes = {"small", "large", "pretranspose"};
  auto run_mode = [&](const std::string &mode, uint32_t store, std::vector<Stage> *stages) {
    DataCopyTiling t = mode == "small" ? small : large;
    t.store = store;
    cudaEvent_t e[3];
    for (auto &ev : e) Check(cudaEventCreate(&ev), "event");
    Check(cudaMemsetAsync(flush.p, 0x5A, flush.n, s), "flush");
    Check(cudaEventRecord(e[0], s), "record");
    if (mode == "small") CheckD(dcopy_datacopy_small(x.p, y.p, &t, ds));
    if (mode == "large") CheckD(dcopy_datacopy_large(x.p, y.p, &t, ds));
    if (mode == "pretranspose") CheckD(dcopy_datacopy_pretranspose(x.p, b.p, &t, ds));
    Check(cudaEventRecord(e[1], s), "record");
    if (mode == "pretranspose") CheckD(dcopy_datacopy_contiguous(b.p, y.p, &t, ds));
    Check(cudaEventRecord(e[2], s), "record");
    Check(cudaEventSynchronize(e[2]), "sync");
    float m1 = 0, m2 = 0;
    Check(cudaEventElapsedTime(&m1, e[0], e[1]), "elapsed");
    Check(cudaEventElapsedTime(&m2, e[1], e[2]), "elapsed");
    if (stages) {
      if (mode == "pretranspose") {
        stages->push_back({"datacopy_pretranspose", m1 * 1e3});
        stages->push_back({"datacopy_contiguous", m2 * 1e3});
      } else {
        stages->push_back({"datacopy_" + mode, m1 * 1e3});
      }
    }
    for (auto &ev : e) cudaEventDestroy(ev);
  };
  // Verification runs: STORE=1, every element checked (asc:149-155).
  for (const auto &mode : modes) {
    Check(cudaMemset(y.p, 0xA5, bytes), "memset");
    run_mode(mode, 1, nullptr);
    Check(cudaMemcpy(output.data(), y.p, bytes, cudaMemcpyDeviceToHost), "D2H");
    for (uint32_t c = 0; c < cols; ++c)
      for (uint32_t r = 0; r < rows; ++r)
        if (output[size_t(c) * rows + r] != input[size_t(r) * cols + c])
          throw std::runtime_error(mode + " verification failed at " + std::to_string(r) + "," +
                                   std::to_string(c));
  }
  // Timed runs: STORE=0 (pretranspose always writes B), rotated order (profile.py:183-186).
  std::map<std::string, std::vector<std::vector<Stage>>> rec;
  for (int trial = 0; trial < trials; ++trial)
    for (int k = 0; k < 3; ++k) {
      const std::string &mode = modes[(trial + k) % 3];
      std::vector<Stage> st;
      run_mode(mode, 0, &st);
      rec[mode].push_back(st);
    }
  std::ostringstream sum;
  std::map<std::string, double> med;
  sum << "{\n  \"metric\": \"device time per workflow (CUDA events; task_duration_us = sum of "
         "the workflow's kernels)\",\n  \"results\": {";
  std::ostringstream raw, stages_csv;
  raw << "mode,trial,rows,cols,tile_cols,tile_bytes,tile_count,task_duration_us\n";
  stages_csv << "mode,trial,kernel,duration_us\n";
  for (size_t mi = 0; mi < modes.size(); ++mi) {
    const std::string &mode = modes[mi];
    const DataCopyTiling &t = mode == "small" ? small : large;
    std::vector<double> total, pre, load;
    for (size_t tr = 0; tr < rec[mode].size(); ++tr) {
      double tot = 0;
      for (const auto &st : rec[mode][tr]) {
        tot += st.us;
        stages_csv << mode << ',' << tr << ',' << st.kernel << ',' << st.us << '\n';
      }
      total.push_back(tot);
      pre.push_back(mode == "pretranspose" ? rec[mode][tr][0].us : 0.0);
      load.push_back(rec[mode][tr].back().us);
      raw << mode << ',' << tr << ',' << rows << ',' << cols << ',' << t.tile_cols << ','
          << t.ub_bytes << ',' << (cols + t.tile_cols - 1) / t.tile_cols << ',' << tot << '\n';
    }
    med[mode] = median(total);
    sum << (mi ? "," : "") << "\n    \"" << mode << "\": {\"task_duration_us\": " << med[mode]
        << ", \"pretranspose_duration_us\": " << median(pre)
        << ", \"load_duration_us\": " << median(load)
        << ", \"min_task_duration_us\": " << *std::min_element(total.begin(), total.end())
        << ", \"max_task_duration_us\": " << *std::max_element(total.begin(), total.end())
        << ", \"GBps\": " << (mode == "pretranspose" ? 3.0 : 1.0) * bytes / (med[mode] * 1e3)
        << "}";
  }
  sum << "\n  },\n  \"small_over_large_duration\": " << med["small"] / med["large"]
      << ",\n  \"pretranspose_over_large_duration\": " << med["pretranspose"] / med["large"]
      << ",\n  \"verification\": \"PASS\"\n}\n";
  std::cout << sum.str();
  if (!outdir.empty()) {
    std::ofstream(outdir + "/summary.json") << sum.str();
    std::ofstream(outdir + "/raw.csv") << raw.str();
    std::ofstream(outdir + "/stages.csv") << stages_csv.str();
    std::ofstream(outdir + "/config.json")
        << "{\"rows\": " << rows << ", \"cols\": " << cols << ", \"small_kib\": " << small_kib
        << ", \"large_kib\": " << large_kib << ", \"trials\": " << trials
        << ", \"device\": " << device << ", \"input_bytes\": " << bytes << "}\n";
  }
  cudaStreamDestroy(s);
  return 0;
}

// ---- nz ---------------------------------------------------------------------------

int run_nz(const Args &a) {
  const int64_t shape[3] = {int64_t(a.num("batch", 16)), int64_t(a.num("h", 4096)),
                            int64_t(a.num("w", 4096))};
  const int reps = int(a.num("reps", 20));
  const double peak = a.num("peak", 6543.4);
  const int64_t c0 = int64_t(a.num("c0", 16));
  const bool zz_format = a.str("format", "nz") == "zz";
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  dcopy_stream_t ds = reinterpret_cast<dcopy_stream_t>(s);
  auto to_frac = zz_format ? dcopy_nd_to_zz : dcopy_nd_to_nz;
  auto to_nd = zz_format ? dcopy_zz_to_nd : dcopy_nz_to_nd;
  int64_t nz[5], hw[3];
  int nz_rank = 0;
  CheckD(zz_format ? dcopy_zz_shape(shape, 3, c0, nz, &nz_rank, hw)
                   : dcopy_nz_shape(shape, 3, c0, nz, &nz_rank, hw));
  uint64_t nd_elems = uint64_t(shape[0]) * shape[1] * shape[2], nz_elems = 1;
  for (int i = 0; i < nz_rank; ++i) nz_elems *= nz[i];
  DevBuf nd(nd_elems * 2), z(nz_elems * 2), back(nd_elems * 2), flush(512ull << 20);
  std::vector<uint16_t> host(nd_elems), host2(nd_elems);
  uint64_t x = 0x9E3779B97F4A7C15ull;  // splitmix64 bit patterns
  for (auto &v : host) {
    x += 0x9E3779B97F4A7C15ull;
    uint64_t z2 = x;
    z2 = (z2 ^ (z2 >> 30)) * 0xBF58476D1CE4E5B9ull;
    z2 = (z2 ^ (z2 >> 27)) * 0x94D049BB133111EBull;
    v = uint16_t(z2 ^ (z2 >> 31));
  }
  Check(cudaMemcpy(nd.p, host.data(), nd_elems * 2, cudaMemcpyHostToDevice), "H2D");
  CheckD(to_frac(z.p, nd.p, shape, 3, 2, c0, ds));
  CheckD(to_nd(back.p, z.p, shape, 3, 2, c0, ds));
  Check(cudaMemcpy(host2.data(), back.p, nd_elems * 2, cudaMemcpyDeviceToHost), "D2H");
  if (std::memcmp(host.data(), host2.data(), nd_elems * 2) != 0)
    throw std::runtime_error("ND -> tiled -> ND round trip differs");
  auto t1 = time_reps([&] { CheckD(to_frac(z.p, nd.p, shape, 3, 2, c0, ds)); }, reps, s, flush);
  auto t2 = time_reps([&] { CheckD(to_nd(back.p, z.p, shape, 3, 2, c0, ds)); }, reps, s, flush);
  const double g1 = double(nd_elems * 2 + nz_elems * 2) / (median(t1) * 1e3);
  const double g2 = double(nd_elems * 2 + nz_elems * 2) / (median(t2) * 1e3);
  const std::string f = zz_format ? "zz" : "nz";
  std::cout << "{\"config\": 4, \"format\": \"" << f << "\", \"c0\": " << c0
            << ", \"shape\": [" << shape[0] << ", " << shape[1] << ", " << shape[2]
            << "], \"nd_to_" << f << "_us\": " << median(t1) << ", \"nd_to_" << f
            << "_GBps\": " << g1 << ", \"" << f << "_to_nd_us\": " << median(t2) << ", \"" << f
            << "_to_nd_GBps\": " << g2
            << ", \"frac_of_peak\": [" << g1 / peak << ", " << g2 / peak
            << "], \"round_trip_bit_exact\": true}" << std::endl;
  cudaStreamDestroy(s);
  return 0;
}

// ---- pcie -------------------------------------------------------------------------

// The copy engine over PCIe as dcopy_copy_ext_staged drives it: the 2-D gather
// host -> device of `rows` bursts of `len` bytes out of `pitch`-byte host rows,
// a contiguous host -> device copy of the same bytes, and the return device ->
// host; each cut into k copies issued back to back on one stream (which shows
// the cost of one copy), then a gather and a return on two streams at once
// (the duplex rate each direction gets).  Host buffers are pinned.  One JSON
// line per case, the median of `reps` timed repetitions.
int run_pcie(const Args &a) {
  const uint64_t rows = uint64_t(a.num("rows", 4096)), len = uint64_t(a.num("len", 4096));
  const uint64_t pitch = uint64_t(a.num("pitch", 16384));
  const int reps = int(a.num("reps", 5));
  if (pitch < len) throw std::runtime_error("pcie: pitch < len");
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  const uint64_t bytes = rows * len;
  void *h_src = nullptr, *h_dst = nullptr;
  Check(cudaHostAlloc(&h_src, rows * pitch, cudaHostAllocDefault), "cudaHostAlloc");
  Check(cudaHostAlloc(&h_dst, bytes, cudaHostAllocDefault), "cudaHostAlloc");
  DevBuf d(bytes), d2(bytes);
  cudaStream_t st[2];
  for (auto &x : st) Check(cudaStreamCreateWithFlags(&x, cudaStreamNonBlocking), "stream");
  cudaEvent_t start, end[2];
  Check(cudaEventCreate(&start), "event");
  for (auto &e : end) Check(cudaEventCreate(&e), "event");
  auto *hs = static_cast<uint8_t *>(h_src);
  auto *hd = static_cast<uint8_t *>(h_dst);
  auto *dd = static_cast<uint8_t *>(d.p);
  auto *dd2 = static_cast<uint8_t *>(d2.p);
  auto gather = [&](int k, cudaStream_t x) {
    const uint64_t per = rows / k;
    for (int i = 0; i < k; ++i)
      Check(cudaMemcpy2DAsync(dd + i * per * len, len, hs + i * per * pitch, pitch, len, per,
                              cudaMemcpyHostToDevice, x), "gather");
  };
  auto h2d = [&](int k, cudaStream_t x) {
    const uint64_t per = bytes / k;
    for (int i = 0; i < k; ++i)
      Check(cudaMemcpyAsync(dd2 + i * per, hs + i * per, per, cudaMemcpyHostToDevice, x), "h2d");
  };
  auto d2h = [&](int k, cudaStream_t x) {
    const uint64_t per = bytes / k;
    for (int i = 0; i < k; ++i)
      Check(cudaMemcpyAsync(hd + i * per, dd + i * per, per, cudaMemcpyDeviceToHost, x), "d2h");
  };
  // Median over reps of the span from `start` (both streams wait on it) to the
  // later of the two streams' end events.
  auto timed = [&](const std::function<void()> &issue) {
    issue();  // warm-up
    Check(cudaDeviceSynchronize(), "sync");
    std::vector<double> us;
    for (int r = 0; r < reps; ++r) {
      Check(cudaEventRecord(start, st[0]), "record");
      Check(cudaStreamWaitEvent(st[1], start, 0), "wait");
      issue();
      for (int i = 0; i < 2; ++i) Check(cudaEventRecord(end[i], st[i]), "record");
      Check(cudaDeviceSynchronize(), "sync");
      double worst = 0;
      for (int i = 0; i < 2; ++i) {
        float ms = 0;
        Check(cudaEventElapsedTime(&ms, start, end[i]), "elapsed");
        worst = std::max(worst, double(ms) * 1e3);
      }
      us.push_back(worst);
    }
    return median(us);
  };
  auto line = [&](const char *name, int k, double us, int directions) {
    std::cout << "{\"pcie\": \"" << name << "\", \"copies\": " << k << ", \"bytes_per_direction\": "
              << bytes << ", \"us\": " << us << ", \"GBps_per_direction\": " << bytes / (us * 1e3)
              << ", \"directions\": " << directions << "}" << std::endl;
  };
  for (int k : {1, 4, 16, 64}) {
    line("gather2d_h2d", k, timed([&] { gather(k, st[0]); }), 1);
    line("contiguous_h2d", k, timed([&] { h2d(k, st[0]); }), 1);
    line("contiguous_d2h", k, timed([&] { d2h(k, st[0]); }), 1);
  }
  line("gather2d_h2d+d2h", 1, timed([&] { gather(1, st[0]); d2h(1, st[1]); }), 2);
  line("contiguous_h2d+d2h", 1, timed([&] { h2d(1, st[0]); d2h(1, st[1]); }), 2);
  cudaEventDestroy(start);
  for (auto &e : end) cudaEventDestroy(e);
  for (auto &x : st) cudaStreamDestroy(x);
  cudaFreeHost(h_src);
  cudaFreeHost(h_dst);
  return 0;
}

// ---- staged ---------------------------------------------------------------------

// BASELINE config 2 end to end from pinned host memory through
// dcopy_copy_ext_staged (copy-engine gather, copy-engine return, 16 MiB device
// staging): `calls` back-to-back calls between CUDA events, the host time spent
// issuing them, and a check of the result; one JSON line per repetition.
int run_staged(const Args &a) {
  const uint32_t rows = 4096, len = 4096, gap = 12288;
  const int calls = int(a.num("calls", 30)), reps = int(a.num("reps", 3));
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  const uint64_t src_bytes = uint64_t(rows) * (len + gap), bytes = uint64_t(rows) * len;
  void *h_src = nullptr, *h_dst = nullptr;
  Check(cudaHostAlloc(&h_src, src_bytes, cudaHostAllocDefault), "cudaHostAlloc");
  Check(cudaHostAlloc(&h_dst, bytes, cudaHostAllocDefault), "cudaHostAlloc");
  auto *hs = static_cast<uint8_t *>(h_src);
  auto *hd = static_cast<uint8_t *>(h_dst);
  for (uint64_t i = 0; i < src_bytes; ++i) hs[i] = uint8_t(i * 131 + (i >> 12));
  DevBuf staging(16ull << 20);
  cudaStream_t s;
  Check(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
  const DcopyExtParams p{rows, len, gap, 0};
  auto call = [&] {
    CheckD(dcopy_copy_ext_staged(h_dst, h_src, &p, staging.p, staging.n,
                                 DCOPY_STAGED_COPY_ENGINE_RETURN,
                                 reinterpret_cast<dcopy_stream_t>(s)));
  };
  for (int w = 0; w < 3; ++w) call();
  Check(cudaStreamSynchronize(s), "sync");
  cudaEvent_t e0, e1;
  Check(cudaEventCreate(&e0), "event");
  Check(cudaEventCreate(&e1), "event");
  for (int r = 0; r < reps; ++r) {
    std::memset(h_dst, 0xA5, bytes);
    Check(cudaEventRecord(e0, s), "record");
    const auto t0 = std::chrono::steady_clock::now();
    for (int c = 0; c < calls; ++c) call();
    const auto t1 = std::chrono::steady_clock::now();
    Check(cudaEventRecord(e1, s), "record");
    Check(cudaEventSynchronize(e1), "sync");
    for (uint32_t row = 0; row < rows; ++row)
      if (std::memcmp(hd + uint64_t(row) * len, hs + uint64_t(row) * (len + gap), len) != 0)
        throw std::runtime_error("staged: result differs at row " + std::to_string(row));
    float ms = 0;
    Check(cudaEventElapsedTime(&ms, e0, e1), "elapsed");
    const double dev_us = double(ms) * 1e3 / calls;
    const double host_us = std::chrono::duration<double, std::micro>(t1 - t0).count() / calls;
    std::cout << "{\"staged\": \"config2\", \"calls\": " << calls << ", \"GBps\": "
              << 2.0 * bytes / (dev_us * 1e3) << ", \"device_us_per_call\": " << dev_us
              << ", \"host_us_per_call\": " << host_us << ", \"verified\": true}" << std::endl;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamDestroy(s);
  cudaFreeHost(h_src);
  cudaFreeHost(h_dst);
  return 0;
}

// ---- fz ---------------------------------------------------------------------------

int run_fz(const Args &a) {
  const int64_t n = int64_t(a.num("n", 2048)), c = int64_t(a.num("c", 2048));
  const int64_t h = int64_t(a.num("h", 3)), w = int64_t(a.num("w", 3));
  const int eb = int(a.num("eb", 2));
  const int64_t c0 = int64_t(a.num("c0", 16));
  const int reps = int(a.num("reps", 20));
  const double peak = a.num("peak", 6543.4);
  // --replay 1: time as bench.py does (graph replay of two alternating weight
  // sets, no L2 eviction) instead of one call per rep after an eviction.
  const bool replay = a.num("replay", 0) != 0;
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  dcopy_stream_t ds = reinterpret_cast<dcopy_stream_t>(s);
  const uint64_t wbytes = uint64_t(n * c * h * w) * eb;
  std::vector<uint8_t> host(wbytes), host2(wbytes);
  uint64_t x = 0x2545F4914F6CDD1Dull;  // xorshift64 bytes
  for (auto &v : host) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    v = uint8_t(x);
  }
  DevBuf src(wbytes), back(wbytes), flush(512ull << 20);
  Check(cudaMemcpy(src.p, host.data(), wbytes, cudaMemcpyHostToDevice), "H2D");
  const struct {
    const char *name;
    int32_t fmt;
    std::vector<int64_t> shape;
  } fmts[] = {{"NCHW", 0, {n, c, h, w}}, {"NHWC", 1, {n, h, w, c}}, {"HWCN", 16, {h, w, c, n}}};
  const std::string wanted = a.str("formats", "nchw,nhwc,hwcn");
  for (const auto &f : fmts) {
    std::string lower(f.name);
    for (auto &ch : lower) ch = char(std::tolower((unsigned char)ch));
    if (wanted.find(lower) == std::string::npos) continue;
    int64_t fz[4];
    CheckD(dcopy_fz_shape(f.fmt, f.shape.data(), 4, c0, 0, fz));
    const uint64_t fbytes = uint64_t(fz[0] * fz[1] * fz[2] * fz[3]) * eb;
    DevBuf z(fbytes);
    CheckD(dcopy_to_fractal_z(z.p, src.p, f.fmt, f.shape.data(), 4, eb, c0, 0, ds));
    CheckD(dcopy_from_fractal_z(back.p, z.p, f.fmt, f.shape.data(), 4, eb, c0, ds));
    Check(cudaMemcpy(host2.data(), back.p, wbytes, cudaMemcpyDeviceToHost), "D2H");
    if (std::memcmp(host.data(), host2.data(), wbytes) != 0)
      throw std::runtime_error(std::string(f.name) + " -> FRACTAL_Z -> back differs");
    double us1 = 0, us2 = 0;
    if (replay) {
      // A second weight / FRACTAL_Z pair (the contents are not checked here).
      DevBuf src2(wbytes), z2(fbytes);
      us1 = replay_us([&] {
        CheckD(dcopy_to_fractal_z(z.p, src.p, f.fmt, f.shape.data(), 4, eb, c0, 0, ds));
        CheckD(dcopy_to_fractal_z(z2.p, src2.p, f.fmt, f.shape.data(), 4, eb, c0, 0, ds));
      }, reps, s) / 2;
      us2 = replay_us([&] {
        CheckD(dcopy_from_fractal_z(back.p, z.p, f.fmt, f.shape.data(), 4, eb, c0, ds));
        CheckD(dcopy_from_fractal_z(src2.p, z2.p, f.fmt, f.shape.data(), 4, eb, c0, ds));
      }, reps, s) / 2;
    } else {
      us1 = median(time_reps(
          [&] { CheckD(dcopy_to_fractal_z(z.p, src.p, f.fmt, f.shape.data(), 4, eb, c0, 0, ds)); },
          reps, s, flush));
      us2 = median(time_reps(
          [&] { CheckD(dcopy_from_fractal_z(back.p, z.p, f.fmt, f.shape.data(), 4, eb, c0, ds)); },
          reps, s, flush));
    }
    const double g1 = double(wbytes + fbytes) / (us1 * 1e3);
    const double g2 = double(wbytes + fbytes) / (us2 * 1e3);
    std::cout << "{\"fz\": \"" << f.name << "\", \"weight_nchw\": [" << n << ", " << c << ", "
              << h << ", " << w << "], \"elem_bytes\": " << eb << ", \"c0\": " << c0
              << ", \"timing\": \"" << (replay ? "graph replay" : "L2 evicted per rep")
              << "\", \"to_fz_us\": " << us1 << ", \"to_fz_GBps\": " << g1
              << ", \"from_fz_us\": " << us2 << ", \"from_fz_GBps\": " << g2
              << ", \"frac_of_peak\": [" << g1 / peak << ", " << g2 / peak
              << "], \"round_trip_bit_exact\": true}" << std::endl;
  }
  cudaStreamDestroy(s);
  return 0;
}

// ---- transpose -----------------------------------------------------------------------

std::vector<int64_t> parse_list(const std::string &text) {
  std::vector<int64_t> v;
  std::stringstream ss(text);
  std::string item;
  while (std::getline(ss, item, ',')) v.push_back(std::stoll(item));
  return v;
}

int run_transpose(const Args &a) {
  const std::vector<int64_t> shape = parse_list(a.str("shape", "32,256,56,56"));
  const std::vector<int64_t> perm = parse_list(a.str("perm", "0,2,3,1"));
  const int eb = int(a.num("eb", 2));
  const int reps = int(a.num("reps", 20));
  const double peak = a.num("peak", 6543.4);
  const int rank = int(shape.size());
  if (perm.size() != shape.size()) throw std::runtime_error("--perm and --shape differ in rank");
  const int32_t dt = eb == 1 ? 4 : eb == 2 ? 1 : eb == 4 ? 0 : eb == 8 ? 9 : 17;
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  dcopy_stream_t ds = reinterpret_cast<dcopy_stream_t>(s);
  uint64_t n = 1;
  for (auto d : shape) n *= uint64_t(d);
  const uint64_t bytes = n * eb;
  std::vector<uint8_t> host(bytes), out(bytes), expect(bytes);
  uint64_t x = 0x9E3779B97F4A7C15ull;
  for (auto &v : host) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    v = uint8_t(x);
  }
  // Host restatement: destination odometer over the permuted shape.
  std::vector<int64_t> heads(rank), dshape(rank), idx(rank, 0);
  for (int i = rank - 1; i >= 0; --i) heads[i] = i == rank - 1 ? 1 : shape[i + 1] * heads[i + 1];
  for (int i = 0; i < rank; ++i) dshape[i] = shape[perm[i]];
  for (uint64_t di = 0; di < n; ++di) {
    int64_t off = 0;
    for (int k = 0; k < rank; ++k) off += idx[k] * heads[perm[k]];
    std::memcpy(&expect[di * eb], &host[off * eb], eb);
    for (int k = rank - 1; k >= 0; --k) {
      if (++idx[k] < dshape[k]) break;
      idx[k] = 0;
    }
  }
  DevBuf src(bytes), dst(bytes), flush(512ull << 20);
  Check(cudaMemcpy(src.p, host.data(), bytes, cudaMemcpyHostToDevice), "H2D");
  CheckD(dcopy_transpose(dst.p, src.p, shape.data(), perm.data(), rank, dt, ds));
  Check(cudaMemcpy(out.data(), dst.p, bytes, cudaMemcpyDeviceToHost), "D2H");
  if (out != expect) throw std::runtime_error("transpose result differs from the host restatement");
  auto t = time_reps(
      [&] { CheckD(dcopy_transpose(dst.p, src.p, shape.data(), perm.data(), rank, dt, ds)); },
      reps, s, flush);
  const double g = 2.0 * bytes / (median(t) * 1e3);
  std::cout << "{\"transpose\": \"" << a.str("shape", "32,256,56,56") << " perm "
            << a.str("perm", "0,2,3,1") << "\", \"elem_bytes\": " << eb
            << ", \"us\": " << median(t) << ", \"GBps\": " << g
            << ", \"frac_of_peak\": " << g / peak << ", \"verified\": true}" << std::endl;
  cudaStreamDestroy(s);
  return 0;
}

// ---- nd -----------------------------------------------------------------------------

// A DataCopyNddma box (dcopy_copy_nd): `sizes` elements, source and destination
// strides from extents padded by --src-pad / --dst-pad elements on every axis but
// the outermost.  Verified element by element (box and untouched gaps).
int run_nd(const Args &a) {
  const std::vector<int64_t> sz = parse_list(a.str("sizes", "64,1024,1024"));
  const int eb = int(a.num("eb", 2));
  const int64_t sp = int64_t(a.num("src-pad", 8)), dp = int64_t(a.num("dst-pad", 0));
  const int reps = int(a.num("reps", 20));
  const double peak = a.num("peak", 6543.4);
  const int nd = int(sz.size());
  const int tma = int(a.num("tma", 0));
  CheckD(dcopy_set_nd_tma(tma, nullptr));
  std::vector<uint64_t> sizes(sz.begin(), sz.end());
  std::vector<int64_t> ss(nd), ds(nd);
  ss[nd - 1] = ds[nd - 1] = 1;
  for (int k = nd - 2; k >= 0; --k) {
    ss[k] = ss[k + 1] * (sz[k + 1] + sp);
    ds[k] = ds[k + 1] * (sz[k + 1] + dp);
  }
  // --src-order: the box axes in the source's memory order, outermost first (an
  // NHWC box of an NCHW tensor is 0,3,1,2); pads apply as above.
  if (a.opt.count("src-order")) {
    const std::vector<int64_t> order = parse_list(a.str("src-order", ""));
    if ((int)order.size() != nd) throw std::runtime_error("--src-order needs one entry per axis");
    int64_t step = 1;
    for (int i = nd - 1; i >= 0; --i) {
      ss[order[i]] = step;
      step *= sz[order[i]] + (i == nd - 1 ? 0 : sp);
    }
  }
  if (a.opt.count("dst-order")) {  // the same for the destination
    const std::vector<int64_t> order = parse_list(a.str("dst-order", ""));
    if ((int)order.size() != nd) throw std::runtime_error("--dst-order needs one entry per axis");
    int64_t step = 1;
    for (int i = nd - 1; i >= 0; --i) {
      ds[order[i]] = step;
      step *= sz[order[i]] + (i == nd - 1 ? 0 : dp);
    }
  }
  uint64_t src_n = 1, dst_n = 1;
  for (int k = 0; k < nd; ++k) {
    src_n += uint64_t(sz[k] - 1) * ss[k];
    dst_n += uint64_t(sz[k] - 1) * ds[k];
  }
  uint64_t n = 1;
  for (auto d : sz) n *= uint64_t(d);
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  dcopy_stream_t dsm = reinterpret_cast<dcopy_stream_t>(s);
  std::vector<uint8_t> host(src_n * eb), out(dst_n * eb);
  uint64_t x = 0x9E3779B97F4A7C15ull;
  for (auto &v : host) {
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    v = uint8_t(x);
  }
  DevBuf src(src_n * eb), dst(dst_n * eb), flush(512ull << 20);
  Check(cudaMemcpy(src.p, host.data(), host.size(), cudaMemcpyHostToDevice), "H2D");
  Check(cudaMemset(dst.p, 0xA5, dst_n * eb), "memset");
  CheckD(dcopy_copy_nd(dst.p, src.p, nd, sizes.data(), ss.data(), ds.data(), eb, dsm));
  Check(cudaMemcpy(out.data(), dst.p, out.size(), cudaMemcpyDeviceToHost), "D2H");
  std::vector<uint8_t> expect(dst_n * eb, 0xA5);
  std::vector<int64_t> idx(nd, 0);
  for (uint64_t e = 0; e < n; ++e) {
    int64_t so = 0, doff = 0;
    for (int k = 0; k < nd; ++k) {
      so += idx[k] * ss[k];
      doff += idx[k] * ds[k];
    }
    std::memcpy(&expect[doff * eb], &host[so * eb], eb);
    for (int k = nd - 1; k >= 0; --k) {
      if (++idx[k] < sz[k]) break;
      idx[k] = 0;
    }
  }
  if (out != expect) throw std::runtime_error("copy_nd result differs from the host restatement");
  auto call = [&] {
    CheckD(dcopy_copy_nd(dst.p, src.p, nd, sizes.data(), ss.data(), ds.data(), eb, dsm));
  };
  auto t = time_reps(call, reps, s, flush);
  auto tg = time_graph_reps(call, reps, s, flush);
  const double host_call_us = host_us_per_call(call, reps, s);
  uint32_t tma_err = 0;
  CheckD(dcopy_tma_error(&tma_err));
  if (tma_err) throw std::runtime_error("TMA box copy gave up a wait");
  const double g = 2.0 * n * eb / (median(t) * 1e3);
  std::cout << "{\"nd\": \"" << a.str("sizes", "64,1024,1024") << "\", \"src_pad\": " << sp
            << ", \"dst_pad\": " << dp << ", \"elem_bytes\": " << eb
            << ", \"tma_selected\": " << (tma ? "true" : "false")
            << ", \"us\": " << median(t) << ", \"GBps\": " << g
            << ", \"frac_of_peak\": " << g / peak << ", \"graph_us\": " << median(tg)
            << ", \"graph_GBps\": " << 2.0 * n * eb / (median(tg) * 1e3)
            << ", \"host_us_per_call\": " << host_call_us << ", \"verified\": true}" << std::endl;
  cudaStreamDestroy(s);
  return 0;
}

// ---- batch ----------------------------------------------------------------------------

// BASELINE config 2's gather (fp32 [4096,4096] cols 1024..2047 -> [4096,1024]) on
// `gathers` independent buffer pairs: one dcopy_copy_ext_batch against one
// dcopy_copy_ext per gather, both verified.
int run_batch(const Args &a) {
  const int gathers = int(a.num("gathers", 16));
  const int reps = int(a.num("reps", 20));
  const double peak = a.num("peak", 6543.4);
  if (gathers < 1 || gathers > 256) throw std::runtime_error("--gathers must be 1..256");
  Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
  cudaStream_t s;
  Check(cudaStreamCreate(&s), "stream");
  dcopy_stream_t ds = reinterpret_cast<dcopy_stream_t>(s);
  const uint32_t rows = 4096, cols = 4096, c0 = 1024, width = 1024;
  const size_t src_bytes = size_t(rows) * cols * 4, dst_bytes = size_t(rows) * width * 4;
  std::vector<std::unique_ptr<DevBuf>> src, dst;
  std::vector<uint32_t> host(size_t(rows) * cols);
  for (size_t i = 0; i < host.size(); ++i) host[i] = uint32_t(i * 2654435761u);
  std::vector<DcopyExtCopy> copies;
  for (int g = 0; g < gathers; ++g) {
    src.push_back(std::make_unique<DevBuf>(src_bytes));
    dst.push_back(std::make_unique<DevBuf>(dst_bytes));
    Check(cudaMemcpy(src.back()->p, host.data(), src_bytes, cudaMemcpyHostToDevice), "H2D");
    Check(cudaMemset(dst.back()->p, 0xA5, dst_bytes), "memset");
    copies.push_back(DcopyExtCopy{dst.back()->p, static_cast<char *>(src.back()->p) + c0 * 4,
                                  DcopyExtParams{rows, width * 4, uint64_t(cols - width) * 4, 0}});
  }
  DevBuf flush(512ull << 20);
  CheckD(dcopy_copy_ext_batch(copies.data(), uint32_t(copies.size()), ds));
  std::vector<uint32_t> out(size_t(rows) * width);
  for (int g = 0; g < gathers; ++g) {
    Check(cudaMemcpy(out.data(), dst[g]->p, dst_bytes, cudaMemcpyDeviceToHost), "D2H");
    for (uint32_t r = 0; r < rows; ++r)
      for (uint32_t c = 0; c < width; ++c)
        if (out[size_t(r) * width + c] != host[size_t(r) * cols + c0 + c])
          throw std::runtime_error("batch gather mismatch");
  }
  auto tb = time_graph_reps([&] { CheckD(dcopy_copy_ext_batch(copies.data(), uint32_t(copies.size()), ds)); },
                            reps, s, flush);
  auto tc = time_graph_reps(
      [&] {
        for (auto &c : copies) CheckD(dcopy_copy_ext(c.dst, c.src, &c.params, ds));
      },
      reps, s, flush);
  const double bytes = 2.0 * dst_bytes * gathers;
  const double gb = bytes / (median(tb) * 1e3), gc = bytes / (median(tc) * 1e3);
  std::cout << "{\"batch\": \"config2 gathers\", \"gathers\": " << gathers
            << ", \"batch_us\": " << median(tb) << ", \"batch_GBps\": " << gb
            << ", \"batch_frac_of_peak\": " << gb / peak << ", \"calls_us\": " << median(tc)
            << ", \"calls_GBps\": " << gc << ", \"calls_frac_of_peak\": " << gc / peak
            << ", \"verified\": true}" << std::endl;
  cudaStreamDestroy(s);
  return 0;
}

// ---- p2p --------------------------------------------------------------------------

int run_p2p(const Args &a) {
  const int dev[2] = {int(a.num("device", 0)), int(a.num("peer", 1))};
  const uint64_t bytes = a.has("kib") ? uint64_t(a.num("kib", 1)) << 10
                                      : uint64_t(a.num("mib", 1024)) << 20;
  const int reps = int(a.num("reps", 5));
  const double peak = a.num("peak", 770.0);  // measured per-direction peer copy
  CheckD(dcopy_enable_peer_access(dev[0], dev[1]));
  CheckD(dcopy_enable_peer_access(dev[1], dev[0]));
  std::unique_ptr<DevBuf> src[2], dst[2];
  cudaStream_t s[2][2];  // [device][0: main, 1: second stream]
  cudaEvent_t ev[2][2][2];
  for (int i = 0; i < 2; ++i) {
    Check(cudaSetDevice(dev[i]), "cudaSetDevice");
    src[i] = std::make_unique<DevBuf>(bytes);
    dst[i] = std::make_unique<DevBuf>(bytes);
    Check(cudaMemset(src[i]->p, 0x11 * (i + 1), bytes), "memset");
    for (int k = 0; k < 2; ++k) {
      Check(cudaStreamCreateWithFlags(&s[i][k], cudaStreamNonBlocking), "stream");
      Check(cudaEventCreate(&ev[i][k][0]), "event");
      Check(cudaEventCreate(&ev[i][k][1]), "event");
    }
  }
  // GPU i sends src[i] to the other GPU's dst.  push: dcopy_p2p_copy on the
  // sender with its automatic engine choice; smpush: the same with the SM
  // engine forced (the bulk-copy push kernel); pull: the load kernel on the
  // receiver; ce: cudaMemcpyPeerAsync; split: SM push of the first half and the
  // copy engine for the second half, on two streams of the sender; pushpull: SM
  // push of the first half on the sender and a pull of the second half on the
  // receiver.
  const uint64_t half = bytes / 2 / 16 * 16;
  auto push = [&](int on, void *d, const void *sp, uint64_t n, int k) {
    Check(cudaSetDevice(dev[on]), "cudaSetDevice");
    CheckD(dcopy_p2p_copy(d, sp, n, reinterpret_cast<dcopy_stream_t>(s[on][k])));
  };
  auto issue = [&](const std::string &mode, int i) {
    const int peer = 1 - i;
    uint8_t *d = static_cast<uint8_t *>(dst[peer]->p);
    const uint8_t *sp = static_cast<const uint8_t *>(src[i]->p);
    if (mode == "push" || mode == "smpush") {
      push(i, d, sp, bytes, 0);
    } else if (mode == "pull") {
      push(peer, d, sp, bytes, 0);
    } else if (mode == "ce") {
      Check(cudaSetDevice(dev[i]), "cudaSetDevice");
      Check(cudaMemcpyPeerAsync(d, dev[peer], sp, dev[i], bytes, s[i][0]), "peer");
    } else if (mode == "split") {
      push(i, d, sp, half, 0);
      Check(cudaMemcpyPeerAsync(d + half, dev[peer], sp + half, dev[i], bytes - half, s[i][1]),
            "peer");
    } else {  // pushpull
      push(i, d, sp, half, 0);
      push(peer, d + half, sp + half, bytes - half, 1);
    }
  };
  auto sync_all = [&] {
    for (int i = 0; i < 2; ++i) {
      Check(cudaSetDevice(dev[i]), "cudaSetDevice");
      Check(cudaDeviceSynchronize(), "sync");
    }
  };
  auto record_all = [&](int which) {
    for (int i = 0; i < 2; ++i) {
      Check(cudaSetDevice(dev[i]), "cudaSetDevice");
      for (int k = 0; k < 2; ++k) Check(cudaEventRecord(ev[i][k][which], s[i][k]), "record");
    }
  };
  std::vector<uint8_t> host(bytes);
  for (const std::string mode : {"push", "smpush", "pull", "ce", "split", "pushpull"}) {
    int32_t prev_engine = 0;
    CheckD(dcopy_set_p2p_engine(mode == "push" ? DCOPY_P2P_ENGINE_AUTO : DCOPY_P2P_ENGINE_SM,
                                &prev_engine));
    for (int senders = 2; senders >= 1; --senders) {
      for (int i = 0; i < 2; ++i) {
        Check(cudaSetDevice(dev[i]), "cudaSetDevice");
        Check(cudaMemset(dst[i]->p, 0, bytes), "memset");
      }
      sync_all();
      for (int w = 0; w < 2; ++w)
        for (int i = 0; i < senders; ++i) issue(mode, i);
      sync_all();
      // Every stream of both GPUs is idle here: the time of the exchange is the
      // longest span between its start and end events.
      record_all(0);
      for (int r = 0; r < reps; ++r)
        for (int i = 0; i < senders; ++i) issue(mode, i);
      record_all(1);
      sync_all();
      double ms = 0;
      for (int i = 0; i < 2; ++i)
        for (int k = 0; k < 2; ++k) {
          float m = 0;
          Check(cudaEventElapsedTime(&m, ev[i][k][0], ev[i][k][1]), "elapsed");
          ms = std::max(ms, double(m));
        }
      uint32_t gave_up = 0;
      for (int i = 0; i < 2; ++i) {
        Check(cudaSetDevice(dev[i]), "cudaSetDevice");
        uint32_t f = 0;
        CheckD(dcopy_p2p_error(&f));
        gave_up |= f;
      }
      for (int i = 0; i < senders; ++i) {
        Check(cudaMemcpy(host.data(), dst[1 - i]->p, bytes, cudaMemcpyDeviceToHost), "D2H");
        const uint8_t want = uint8_t(0x11 * (i + 1));
        if (gave_up || std::any_of(host.begin(), host.end(), [&](uint8_t v) { return v != want; }))
          throw std::runtime_error("p2p " + mode + ": received bytes differ");
      }
      const double gbps = double(bytes) * reps / (ms * 1e6);
      std::cout << "{\"p2p\": \"" << mode << "\", \"senders\": " << senders
                << ", \"bytes_per_sender\": " << bytes << ", \"GBps_per_direction\": " << gbps
                << ", \"frac_of_peer_copy\": " << gbps / peak << ", \"verified\": true}"
                << std::endl;
    }
    CheckD(dcopy_set_p2p_engine(prev_engine, nullptr));
  }
  for (int i = 0; i < 2; ++i) {
    Check(cudaSetDevice(dev[i]), "cudaSetDevice");
    for (int k = 0; k < 2; ++k) {
      cudaEventDestroy(ev[i][k][0]);
      cudaEventDestroy(ev[i][k][1]);
      cudaStreamDestroy(s[i][k]);
    }
    src[i].reset();
    dst[i].reset();
  }
  return 0;
}

}  // namespace

int main(int argc, char **argv) {
  try {
    if (argc < 2) throw std::runtime_error("usage: dcopy_bench sweep|standalone|nz|fz|transpose|nd|batch|p2p|pcie|staged [options]");
    const std::string cmd = argv[1];
    Args a(argc, argv);
    // --l2-fetch B: the context's L2 fetch-granularity hint (cudaLimitMaxL2FetchGranularity,
    // 0..128 bytes) for every command; it lasts as long as this process.
    if (a.opt.count("l2-fetch")) {
      Check(cudaSetDevice(int(a.num("device", 0))), "cudaSetDevice");
      Check(cudaDeviceSetLimit(cudaLimitMaxL2FetchGranularity, size_t(a.num("l2-fetch", 64))),
            "cudaDeviceSetLimit");
      size_t got = 0;
      Check(cudaDeviceGetLimit(&got, cudaLimitMaxL2FetchGranularity), "cudaDeviceGetLimit");
      std::cerr << "L2 fetch granularity limit: " << got << " bytes\n";
    }
    if (cmd == "sweep") return run_sweep(a);
    if (cmd == "standalone") return run_standalone(a);
    if (cmd == "nz") return run_nz(a);
    if (cmd == "p2p") return run_p2p(a);
    if (cmd == "fz") return run_fz(a);
    if (cmd == "pcie") return run_pcie(a);
    if (cmd == "staged") return run_staged(a);
    if (cmd == "transpose") return run_transpose(a);
    if (cmd == "nd") return run_nd(a);
    if (cmd == "batch") return run_batch(a);
    throw std::runtime_error("unknown command " + cmd);
  } catch (const std::exception &e) {
    std::cerr << "dcopy_bench: " << e.what() << '\n';
    return 1;
  }
}
