// GPU check of the numerics gate's failure path.  The reference tests its gate
// with a deliberately nondeterministic op (tests/test_graph_host.cpp:1558 of
// the reference); this does the same against GraphExecutor::validate_numerics:
//   * an op whose output changes on every launch (a byte fill with a launch
//     counter) must make the gate fail and name the tensor it compared;
//   * the same graph with a deterministic op (a device-to-device copy) passes.
// Both ops are defined here, outside the library.  One GPU.
// Prints "OK" and exits 0, or prints the failed check and exits 1.
#include <cuda_runtime.h>

#include <cstdio>
#include <memory>
#include <string>
#include <vector>

#include "mcke/graph/executor.hpp"

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED line %d: %s\n", __LINE__, #c);           \
      return 1;                                                    \
    }                                                              \
  } while (0)

namespace {

using namespace mcke;

Status from_cuda(cudaError_t e) {
  return e == cudaSuccess ? OkStatus() : Status(StatusCode::kCudaError, cudaGetErrorString(e));
}

// Same shape and dtype out as in.
class ElementwiseTestOp : public Op {
 public:
  [[nodiscard]] StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>& in) const override {
    if (in.size() != 1) return InvalidArgumentError("one input");
    TensorDesc d;
    d.shape = in[0].shape;
    d.dtype = in[0].dtype;
    return std::vector<TensorDesc>{d};
  }
  [[nodiscard]] OpCost cost(const std::vector<TensorDesc>&) const override { return {}; }
};

// Deliberately nondeterministic: every launch fills its output with a
// different byte (the launch count), whatever the input.
class CounterFillOp final : public ElementwiseTestOp {
 public:
  [[nodiscard]] std::string_view type_name() const override { return "CounterFill"; }
  [[nodiscard]] Status launch(const OpContext& ctx, const std::vector<Tensor>&,
                              const std::vector<Tensor>& out) override {
    ++launches_;
    return from_cuda(cudaMemsetAsync(out[0].data, launches_ & 0xFF, out[0].nbytes(),
                                     static_cast<cudaStream_t>(ctx.stream)));
  }

 private:
  int launches_ = 0;
};

// Deterministic: a device-to-device copy of the input.
class CopyOp final : public ElementwiseTestOp {
 public:
  [[nodiscard]] std::string_view type_name() const override { return "Copy"; }
  [[nodiscard]] Status launch(const OpContext& ctx, const std::vector<Tensor>& in,
                              const std::vector<Tensor>& out) override {
    return from_cuda(cudaMemcpyAsync(out[0].data, in[0].data, in[0].nbytes(), cudaMemcpyDeviceToDevice,
                                     static_cast<cudaStream_t>(ctx.stream)));
  }
};

// x -> op -> y, with x set from the host; returns the gate's verdict.
StatusOr<NumericsResult> gate(OpPtr op) {
  Graph g;
  TensorDesc xd;
  xd.shape = Shape{64, 256};
  xd.dtype = DType::kF32;
  xd.name = "x";
  const TensorId x = g.add_input(xd);
  auto y = g.add_node("under_test", std::move(op), {x});
  MCKE_RETURN_IF_ERROR(y.status());
  MCKE_RETURN_IF_ERROR(g.mark_output((*y)[0]));
  MCKE_RETURN_IF_ERROR(g.finalize());
  ExecutorOptions o;
  o.num_streams = 2;
  o.validate_numerics = true;
  GraphExecutor ex(g, o);
  MCKE_RETURN_IF_ERROR(ex.plan());
  std::vector<float> host(64 * 256);
  for (std::size_t i = 0; i < host.size(); ++i) host[i] = static_cast<float>(i % 97) * 0.5f;
  MCKE_RETURN_IF_ERROR(ex.set_input(x, host.data(), host.size() * sizeof(float)));
  return ex.validate_numerics(3);
}

}  // namespace

int main() {
  auto bad = gate(std::make_unique<CounterFillOp>());
  if (!bad.ok()) std::printf("gate call failed: %s\n", bad.status().message().c_str());
  CHECK(bad.ok());
  CHECK(!bad->passed);
  CHECK(bad->detail.find("word") != std::string::npos);
  std::printf("nondeterministic op: %s\n", bad->detail.c_str());

  auto good = gate(std::make_unique<CopyOp>());
  if (!good.ok()) std::printf("gate call failed: %s\n", good.status().message().c_str());
  CHECK(good.ok());
  if (!good->passed) std::printf("%s\n", good->detail.c_str());
  CHECK(good->passed);
  CHECK(good->configs_compared > 1);
  std::printf("OK\n");
  return 0;
}
