// qconv_bench: the reference's conv_bench driver pattern (src/main.cpp:76-120, 292-335) for the
// quantized path, calling the B200 kernels.
//
// Built against the reference's own headers and its src/bench.cpp (benchmark_cuda_op,
// src/bench.cpp:8-45), src/cuda_utils.cpp (CudaEventTimer) and src/cpu_ref.cpp (the CPU checker),
// compiled from their sources, and linked with libb200q_refshim.so + libb200q.so:
//   --op qfprop  times launch_fprop_nhwc_qi32<Tin> / launch_block_fprop_nhwc_qi32<Tin>, the
//                reference's own template entry points (src/conv_types.h:308-340), which reach the
//                shim's conv_quant_detail symbols, on float codes with per-image zero points;
//   --op s8      times b200q_conv2d_s8 (int8 tensors, int32 accumulators or the requantized int8
//                output) through the C ABI;
//   --check      compares every output element with cpu_fprop_nhwc_qi32 / cpu_block_fprop_nhwc_qi32
//                (exact int32 equality, the compare of quant_conv_test.cu:96-112).
// Output lines follow print_bench / print_verify of src/main.cpp; the last line is
// "qconv_bench PASS" when every check passed.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdlib>
#include <iomanip>
#include <iostream>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "b200q.h"
#include "conv_types.h"
#include "cuda_utils.h"

namespace {

using nnalgebra::DataType;

struct Options {
  std::string op = "all";            // qfprop | s8 | all
  std::string qtype = "u8";          // u8 | s5
  std::string custom_mode = "explicit";  // explicit | blocked
  int n = 1, h = 56, w = 56, c = 64, k = 64, r = 3, s = 3;
  int pad_h = 1, pad_w = 1, stride_h = 1, stride_w = 1, dilation_h = 1, dilation_w = 1, groups = 1;
  int block_by = 1, block_bx = 1;
  int warmup = 5, iters = 20;
  uint32_t seed = 42;
  bool check = false;
  bool bench_suite = false;
};

struct Case {
  std::string name;
  int n, h, w, c, k, r, s, pad_h, pad_w, stride_h, stride_w, dilation_h, dilation_w, groups, block_by, block_bx;
};

int parse_int(const std::string& v, const char* what) {
  try {
    size_t pos = 0;
    const int x = std::stoi(v, &pos);
    if (pos != v.size()) throw std::invalid_argument(v);
    return x;
  } catch (const std::exception&) {
    throw std::runtime_error(std::string("bad integer for ") + what + ": " + v);
  }
}

Options parse_args(int argc, char** argv) {
  Options o;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto val = [&](const char* name) -> std::string {
      if (i + 1 >= argc) throw std::runtime_error(std::string("missing value for ") + name);
      return argv[++i];
    };
    if (a == "--op") o.op = val("--op");
    else if (a == "--qtype") o.qtype = val("--qtype");
    else if (a == "--custom_mode") o.custom_mode = val("--custom_mode");
    else if (a == "--n") o.n = parse_int(val("--n"), "--n");
    else if (a == "--h") o.h = parse_int(val("--h"), "--h");
    else if (a == "--w") o.w = parse_int(val("--w"), "--w");
    else if (a == "--c") o.c = parse_int(val("--c"), "--c");
    else if (a == "--k") o.k = parse_int(val("--k"), "--k");
    else if (a == "--r") o.r = parse_int(val("--r"), "--r");
    else if (a == "--s") o.s = parse_int(val("--s"), "--s");
    else if (a == "--pad_h") o.pad_h = parse_int(val("--pad_h"), "--pad_h");
    else if (a == "--pad_w") o.pad_w = parse_int(val("--pad_w"), "--pad_w");
    else if (a == "--stride_h") o.stride_h = parse_int(val("--stride_h"), "--stride_h");
    else if (a == "--stride_w") o.stride_w = parse_int(val("--stride_w"), "--stride_w");
    else if (a == "--dilation_h") o.dilation_h = parse_int(val("--dilation_h"), "--dilation_h");
    else if (a == "--dilation_w") o.dilation_w = parse_int(val("--dilation_w"), "--dilation_w");
    else if (a == "--groups") o.groups = parse_int(val("--groups"), "--groups");
    else if (a == "--block_by") o.block_by = parse_int(val("--block_by"), "--block_by");
    else if (a == "--block_bx") o.block_bx = parse_int(val("--block_bx"), "--block_bx");
    else if (a == "--warmup") o.warmup = parse_int(val("--warmup"), "--warmup");
    else if (a == "--iters") o.iters = parse_int(val("--iters"), "--iters");
    else if (a == "--seed") o.seed = static_cast<uint32_t>(parse_int(val("--seed"), "--seed"));
    else if (a == "--check") o.check = true;
    else if (a == "--bench_suite") o.bench_suite = true;
    else if (a == "--help") {
      std::cout << "qconv_bench options:\n"
                << "  --op qfprop|s8|all  --qtype u8|s5  --custom_mode explicit|blocked\n"
                << "  --n --h --w --c --k --r --s\n"
                << "  --pad_h --pad_w --stride_h --stride_w --dilation_h --dilation_w --groups\n"
                << "  --block_by --block_bx  --warmup --iters --seed  --check --bench_suite\n";
      std::exit(0);
    } else {
      throw std::runtime_error("unknown argument: " + a);
    }
  }
  if (o.op != "qfprop" && o.op != "s8" && o.op != "all") throw std::runtime_error("--op must be qfprop|s8|all");
  if (o.qtype != "u8" && o.qtype != "s5") throw std::runtime_error("--qtype must be u8|s5");
  if (o.custom_mode != "explicit" && o.custom_mode != "blocked")
    throw std::runtime_error("--custom_mode must be explicit|blocked");
  return o;
}

// The reference's conv_bench suite geometry (src/main.cpp:163-186) and the BASELINE shapes of the
// int8 path.
std::vector<Case> bench_suite(bool blocked) {
  if (blocked)
    return {{"blocked_resnet_56x56_b2x2", 32, 56, 56, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 2, 2},
            {"blocked_resnet_28x28_b2x4", 32, 28, 28, 128, 256, 3, 3, 1, 1, 1, 1, 1, 1, 1, 2, 4},
            {"blocked_pointwise_1x1_b4x4", 32, 56, 56, 128, 256, 1, 1, 0, 0, 1, 1, 1, 1, 1, 4, 4}};
  return {{"resnet_like_56x56", 32, 56, 56, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1},
          {"resnet_like_28x28", 32, 28, 28, 128, 256, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1},
          {"downsample_stride2", 32, 112, 112, 32, 32, 3, 3, 1, 1, 2, 2, 1, 1, 1, 1, 1},
          {"depthwise_3x3", 32, 56, 56, 128, 128, 3, 3, 1, 1, 1, 1, 1, 1, 128, 1, 1},
          {"grouped_g4", 32, 56, 56, 128, 128, 3, 3, 1, 1, 1, 1, 1, 1, 4, 1, 1},
          {"pointwise_1x1", 32, 56, 56, 128, 256, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1, 1},
          {"dilated_3x3", 16, 64, 64, 64, 64, 3, 3, 2, 2, 1, 1, 2, 2, 1, 1, 1},
          {"small_batch", 1, 56, 56, 64, 64, 3, 3, 1, 1, 1, 1, 1, 1, 1, 1, 1},
          {"config4a_pointwise_b64", 64, 14, 14, 1024, 2048, 1, 1, 0, 0, 1, 1, 1, 1, 1, 1, 1}};
}

void print_bench(const std::string& tag, const BenchResult& b) {
  std::cout << std::fixed << std::setprecision(3) << tag << " median=" << b.median_ms << " ms"
            << " p90=" << b.p90_ms << " ms"
            << " gflops=" << b.gflops << "\n";
}

template <typename T>
struct Dev {
  T* ptr = nullptr;
  explicit Dev(size_t count) { CUDA_CHECK(cudaMalloc(&ptr, count * sizeof(T) + 16)); }
  ~Dev() { cudaFree(ptr); }
  Dev(const Dev&) = delete;
  Dev& operator=(const Dev&) = delete;
};

size_t count_mismatches(const std::vector<int32_t>& ref, const std::vector<int32_t>& got) {
  if (ref.size() != got.size()) return ref.size() + got.size();
  size_t bad = 0;
  for (size_t i = 0; i < ref.size(); ++i) bad += ref[i] != got[i];
  return bad;
}

void print_check(const std::string& tag, size_t bad, size_t total, bool& all_ok) {
  std::cout << tag << " pass=" << (bad == 0 ? "yes" : "no") << " mismatches=" << bad << " of " << total << "\n";
  all_ok = all_ok && bad == 0;
}

template <DataType Tin>
std::vector<nnalgebra::QuantizationParameters<Tin>> input_qparams(int n, std::mt19937& gen);
template <>
std::vector<nnalgebra::QuantizationParameters<DataType::LinQuantU8>> input_qparams(int n, std::mt19937& gen) {
  std::vector<nnalgebra::QuantizationParameters<DataType::LinQuantU8>> v(n);
  for (auto& q : v) q.zero_point = static_cast<uint8_t>(gen() % 256);
  return v;
}
template <>
std::vector<nnalgebra::QuantizationParameters<DataType::LinQuantS5>> input_qparams(int n, std::mt19937& gen) {
  std::vector<nnalgebra::QuantizationParameters<DataType::LinQuantS5>> v(n);
  for (auto& q : v) q.zero_point = static_cast<int8_t>(static_cast<int>(gen() % 31) - 15);
  return v;
}

// Quantized conv through the reference's own template entry points (float codes, zero points).
template <DataType Tin>
void run_qfprop(const Options& o, const Case& bc, bool blocked, bool& all_ok) {
  using QP = nnalgebra::QuantizationParameters<Tin>;
  std::mt19937 gen(o.seed);
  const bool u8 = Tin == DataType::LinQuantU8;
  auto code = [&]() { return static_cast<float>(u8 ? static_cast<int>(gen() % 256) : static_cast<int>(gen() % 31) - 15); };
  Conv2DParams p;
  p.pad_h = bc.pad_h; p.pad_w = bc.pad_w; p.stride_h = bc.stride_h; p.stride_w = bc.stride_w;
  p.dilation_h = bc.dilation_h; p.dilation_w = bc.dilation_w; p.groups = bc.groups;
  BlockConv2DParams bp;
  bp.conv = p;
  bp.block_by = bc.block_by;
  bp.block_bx = bc.block_bx;
  TensorNHWC x(bc.n, bc.h, bc.w, bc.c);
  for (float& v : x.data) v = code();
  const int cg = bc.c / bc.groups;
  FilterKRSC w(bc.r, bc.s, cg, bc.k);
  BlockFilterKByBxRSC wb(bc.k, bc.block_by, bc.block_bx, bc.r, bc.s, cg);
  std::vector<float>& wdata = blocked ? wb.data : w.data;
  for (float& v : wdata) v = code();
  const std::vector<QP> in_qp = input_qparams<Tin>(bc.n, gen);
  QP f_qp;
  f_qp.zero_point = u8 ? static_cast<decltype(f_qp.zero_point)>(gen() % 256)
                       : static_cast<decltype(f_qp.zero_point)>(static_cast<int>(gen() % 31) - 15);
  const ConvShape sh = infer_conv_shape(x, w, p);
  const size_t y_count = static_cast<size_t>(bc.n) * sh.ho * sh.wo * bc.k;
  Dev<float> d_x(x.elements()), d_w(wdata.size());
  Dev<int32_t> d_y(y_count);
  Dev<QP> d_in(in_qp.size()), d_f(1);
  CUDA_CHECK(cudaMemcpy(d_x.ptr, x.ptr(), x.elements() * sizeof(float), cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_w.ptr, wdata.data(), wdata.size() * sizeof(float), cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_in.ptr, in_qp.data(), in_qp.size() * sizeof(QP), cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_f.ptr, &f_qp, sizeof(QP), cudaMemcpyHostToDevice));
  const size_t flops = 2ull * bc.n * sh.ho * sh.wo * bc.r * bc.s * cg * bc.k;
  BenchResult b = benchmark_cuda_op("qfprop", o.warmup, o.iters, flops, [&]() {
    if (blocked)
      launch_block_fprop_nhwc_qi32<Tin>(d_x.ptr, d_w.ptr, d_y.ptr, bc.n, bc.h, bc.w, bc.c, bc.r, bc.s, bc.k, bp,
                                        d_in.ptr, d_f.ptr);
    else
      launch_fprop_nhwc_qi32<Tin>(d_x.ptr, d_w.ptr, d_y.ptr, bc.n, bc.h, bc.w, bc.c, bc.r, bc.s, bc.k, p, d_in.ptr,
                                  d_f.ptr);
  });
  CUDA_CHECK(cudaDeviceSynchronize());
  print_bench(std::string("custom qfprop ") + o.qtype + (blocked ? " blocked" : ""), b);
  std::cout << "path " << b200q_last_path() << "\n";
  if (o.check) {
    std::vector<int32_t> got(y_count);
    CUDA_CHECK(cudaMemcpy(got.data(), d_y.ptr, y_count * sizeof(int32_t), cudaMemcpyDeviceToHost));
    TensorNHWCI32 ref;
    if (blocked)
      cpu_block_fprop_nhwc_qi32<Tin>(x, wb, bp, ref, in_qp.data(), &f_qp);
    else
      cpu_fprop_nhwc_qi32<Tin>(x, w, p, ref, in_qp.data(), &f_qp);
    print_check("check qfprop custom_vs_cpu", count_mismatches(ref.data, got), y_count, all_ok);
  }
}

// int8 conv through the C ABI: int32 accumulators (checked) and the requantized int8 output (timed).
void run_s8(const Options& o, const Case& bc, bool& all_ok) {
  std::mt19937 gen(o.seed + 1);
  Conv2DParams p;
  p.pad_h = bc.pad_h; p.pad_w = bc.pad_w; p.stride_h = bc.stride_h; p.stride_w = bc.stride_w;
  p.dilation_h = bc.dilation_h; p.dilation_w = bc.dilation_w; p.groups = bc.groups;
  const b200q_conv_params cp{p.pad_h, p.pad_w, p.stride_h, p.stride_w, p.dilation_h, p.dilation_w, p.groups};
  const int cg = bc.c / bc.groups;
  TensorNHWC x(bc.n, bc.h, bc.w, bc.c);
  FilterKRSC w(bc.r, bc.s, cg, bc.k);
  std::vector<int8_t> x8(x.elements()), w8(w.elements());
  for (size_t i = 0; i < x8.size(); ++i) {
    x8[i] = static_cast<int8_t>(static_cast<int>(gen() % 255) - 127);
    x.data[i] = x8[i];
  }
  for (size_t i = 0; i < w8.size(); ++i) {
    w8[i] = static_cast<int8_t>(static_cast<int>(gen() % 255) - 127);
    w.data[i] = w8[i];
  }
  std::vector<int32_t> bias(bc.k);
  std::vector<float> scale(bc.k);
  for (int i = 0; i < bc.k; ++i) {
    bias[i] = static_cast<int32_t>(gen() % 65537) - 32768;
    scale[i] = 1e-4f + 9e-4f * static_cast<float>(gen() % 10000) / 10000.0f;
  }
  const ConvShape sh = infer_conv_shape(x, w, p);
  const size_t y_count = static_cast<size_t>(bc.n) * sh.ho * sh.wo * bc.k;
  Dev<int8_t> d_x(x8.size()), d_w(w8.size()), d_y8(y_count);
  Dev<int32_t> d_y(y_count), d_b(bc.k);
  Dev<float> d_s(bc.k);
  CUDA_CHECK(cudaMemcpy(d_x.ptr, x8.data(), x8.size(), cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_w.ptr, w8.data(), w8.size(), cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_b.ptr, bias.data(), bc.k * sizeof(int32_t), cudaMemcpyHostToDevice));
  CUDA_CHECK(cudaMemcpy(d_s.ptr, scale.data(), bc.k * sizeof(float), cudaMemcpyHostToDevice));
  const size_t flops = 2ull * bc.n * sh.ho * sh.wo * bc.r * bc.s * cg * bc.k;
  const b200q_epilogue e32{B200Q_OUT_S32, 0, 0, 0};
  const b200q_epilogue e8{B200Q_OUT_S8, 0, 0, 127};  // bias + scale + ReLU
  auto call = [&](const b200q_epilogue& e, void* y, const int32_t* b, const float* s) {
    const int rc = b200q_conv2d_s8(d_x.ptr, d_w.ptr, b, s, y, bc.n, bc.h, bc.w, bc.c, bc.r, bc.s, bc.k, &cp, &e,
                                   nullptr);
    if (rc != B200Q_OK) throw std::runtime_error(std::string("b200q_conv2d_s8: ") + b200q_last_error());
  };
  BenchResult b32 = benchmark_cuda_op("s8", o.warmup, o.iters, flops, [&]() { call(e32, d_y.ptr, nullptr, nullptr); });
  print_bench("custom s8 int32-out", b32);
  std::cout << "path " << b200q_last_path() << "\n";
  BenchResult b8 = benchmark_cuda_op("s8", o.warmup, o.iters, flops, [&]() { call(e8, d_y8.ptr, d_b.ptr, d_s.ptr); });
  print_bench("custom s8 int8-out relu", b8);
  if (o.check) {
    std::vector<int32_t> got(y_count);
    CUDA_CHECK(cudaMemcpy(got.data(), d_y.ptr, y_count * sizeof(int32_t), cudaMemcpyDeviceToHost));
    using QP = nnalgebra::QuantizationParameters<DataType::LinQuantS5>;
    std::vector<QP> zin(bc.n);
    QP zf;
    TensorNHWCI32 ref;
    cpu_fprop_nhwc_qi32<DataType::LinQuantS5>(x, w, p, ref, zin.data(), &zf);
    print_check("check s8 custom_vs_cpu", count_mismatches(ref.data, got), y_count, all_ok);
  }
}

}  // namespace

int main(int argc, char** argv) {
  try {
    const Options o = parse_args(argc, argv);
    const bool blocked = o.custom_mode == "blocked";
    std::vector<Case> cases;
    if (o.bench_suite) {
      cases = bench_suite(blocked);
    } else {
      cases.push_back({"cli", o.n, o.h, o.w, o.c, o.k, o.r, o.s, o.pad_h, o.pad_w, o.stride_h, o.stride_w,
                       o.dilation_h, o.dilation_w, o.groups, o.block_by, o.block_bx});
    }
    bool all_ok = true;
    for (const Case& bc : cases) {
      std::cout << "case " << bc.name << " n=" << bc.n << " h=" << bc.h << " w=" << bc.w << " c=" << bc.c
                << " k=" << bc.k << " r=" << bc.r << " s=" << bc.s << " stride=" << bc.stride_h << "x" << bc.stride_w
                << " pad=" << bc.pad_h << "x" << bc.pad_w << " dilation=" << bc.dilation_h << "x" << bc.dilation_w
                << " groups=" << bc.groups;
      if (blocked) std::cout << " blocks=" << bc.block_by << "x" << bc.block_bx;
      std::cout << "\n";
      if (o.op == "qfprop" || o.op == "all") {
        if (o.qtype == "u8")
          run_qfprop<DataType::LinQuantU8>(o, bc, blocked, all_ok);
        else
          run_qfprop<DataType::LinQuantS5>(o, bc, blocked, all_ok);
      }
      if ((o.op == "s8" || o.op == "all") && !blocked) run_s8(o, bc, all_ok);
    }
    if (!o.check) {
      std::cout << "qconv_bench done (no --check)\n";
      return 0;
    }
    std::cout << (all_ok ? "qconv_bench PASS" : "qconv_bench FAIL") << "\n";
    return all_ok ? 0 : 1;
  } catch (const std::exception& ex) {
    std::cerr << "error: " << ex.what() << "\n";
    return 2;
  }
}
