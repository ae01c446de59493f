// rustorch_b200.hpp — C++ mirror of RusTorch's operator interface for the
// dense-contraction path, running on the B200 backend (librustorch_b200.so).
//
// Same names, argument meaning and error behaviour as the Rust API it stands
// in for (paths relative to the RusTorch project root):
//   Tensor::new / matmul / conv2d / relu / add / t      rustorch-core/src/tensor.rs
//   ops::matmul                                         rustorch-core/src/ops.rs:1888
//   ops::matmul_fused + backend::Activation             rustorch-core/src/ops.rs:1543,
//                                                       rustorch-core/src/backend/mod.rs:1-7
//   ops::conv2d                                         rustorch-core/src/ops/conv.rs:738
//   ops::max_pool2d                                     rustorch-core/src/ops/pool.rs:115
//   nn::Module / nn::Linear / nn::Conv2d                rustorch-nn/src/{module,linear,conv}.rs
//   jit::{NodeType, Graph, Optimizer, Executor}         rustorch-core/src/jit.rs
// A Rust panic ("Matmul only supports 2D", "Matmul dimension mismatch", ...)
// is a rustorch::Panic exception carrying the same message.
//
// Device semantics: tensors live on the CPU or on a CUDA device.  An op whose
// inputs are all CUDA tensors runs on that device and returns a CUDA tensor;
// an op whose inputs are all CPU tensors (what existing RusTorch callers pass)
// copies them to the device, runs there, and returns a CPU tensor — callers
// change nothing.  There is no CPU compute path.
#pragma once

#include <rustorch_b200.h>

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

namespace rustorch {

struct Panic : std::runtime_error {
  using std::runtime_error::runtime_error;
};

// backend::Activation (rustorch-core/src/backend/mod.rs:1-7).
enum class Activation : int { None = 0, ReLU = 1, Sigmoid = 2, Tanh = 3 };

struct Device {
  enum Kind { Cpu, Cuda };
  Kind kind = Cpu;
  int index = 0;
  static Device cpu() { return Device{Cpu, 0}; }
  static Device cuda(int i = 0) { return Device{Cuda, i}; }
  bool is_cuda() const { return kind == Cuda; }
  bool operator==(const Device& o) const { return kind == o.kind && (kind == Cpu || index == o.index); }
  bool operator!=(const Device& o) const { return !(*this == o); }
};

// Backend state: one rtb_ctx per device (created on first use), the contraction
// precision used by ops (RTB_PREC_3XTF32 by default), and device sync.
rtb_ctx* context(int device);
void set_precision(int precision);
int precision();
// Waits for the device and turns a device-side timeout into a Panic.
void synchronize(int device);

// Host <-> device tensor copies made so far by this process (Tensor::to and
// the ops' staging of CPU operands); diagnostics for keeping data resident.
uint64_t transfer_count();

using Pair = std::pair<size_t, size_t>;

class Tensor {
 public:
  Tensor() = default;
  // Tensor::new(&data, &shape) (rustorch-core/src/tensor.rs)
  static Tensor new_(const std::vector<float>& data, const std::vector<size_t>& shape);
  static Tensor zeros(const std::vector<size_t>& shape, Device d = Device::cpu());
  static Tensor ones(const std::vector<size_t>& shape, Device d = Device::cpu());
  static Tensor full(const std::vector<size_t>& shape, float v, Device d = Device::cpu());
  // Seeded synthetic data from the backend's SplitMix64 generator.
  static Tensor randn(const std::vector<size_t>& shape, uint64_t seed, uint64_t tensor_id,
                      float mean = 0.f, float std_dev = 1.f, Device d = Device::cpu());
  static Tensor uniform(const std::vector<size_t>& shape, uint64_t seed, uint64_t tensor_id,
                        float lo, float hi, Device d = Device::cpu());
  // An uninitialised contiguous tensor on `d` (device memory from the backend pool).
  static Tensor empty(const std::vector<size_t>& shape, Device d);

  const std::vector<size_t>& shape() const { return shape_; }
  const std::vector<size_t>& strides() const { return strides_; }
  size_t dim() const { return shape_.size(); }
  size_t numel() const;
  bool defined() const { return static_cast<bool>(storage_); }
  bool is_contiguous() const;
  Device device() const;

  // Host copy of the elements in logical (row-major) order.  Like the
  // reference's Storage::data on non-CPU storage, panics for a CUDA tensor:
  // move it with to_cpu() first.
  std::vector<float> data() const;
  Tensor to(Device d) const;
  Tensor to_cpu() const { return to(Device::cpu()); }
  Tensor to_cuda(int i = 0) const { return to(Device::cuda(i)); }

  Tensor t() const;  // transpose view of a 2-D tensor (no copy)
  Tensor permute(const std::vector<size_t>& dims) const;
  Tensor contiguous() const;
  Tensor reshape(const std::vector<size_t>& shape) const;

  Tensor matmul(const Tensor& rhs) const;
  Tensor conv2d(const Tensor& weight, Pair stride, Pair padding) const;
  Tensor relu() const;
  Tensor add(const Tensor& rhs) const;
  Tensor mul(const Tensor& rhs) const;

  // Raw element pointer (storage base + view offset) of a CUDA tensor.
  const float* device_ptr() const;
  float* device_ptr();

  struct Storage;

 private:
  std::shared_ptr<Storage> storage_;
  std::vector<size_t> shape_, strides_;
  size_t offset_ = 0;
  friend struct TensorAccess;
};

namespace ops {
Tensor matmul(const Tensor& lhs, const Tensor& rhs);
Tensor matmul_fused(const Tensor& lhs, const Tensor& rhs, const Tensor* bias, Activation act);
// ops::matmul_bias_norm_activation (rustorch-core/src/ops.rs:1815-1886):
// act(layer_norm(lhs.matmul(rhs) + bias, [n], norm_weight, norm_bias, eps)).
Tensor matmul_bias_norm_activation(const Tensor& lhs, const Tensor& rhs, const Tensor* bias,
                                   const Tensor* norm_weight, const Tensor* norm_bias, float eps,
                                   Activation act);
Tensor conv2d(const Tensor& input, const Tensor& weight, Pair stride, Pair padding);
// One fused kernel: act(conv2d(input, weight) + bias[c] + residual).
Tensor conv2d_fused(const Tensor& input, const Tensor& weight, const Tensor* bias, Pair stride,
                    Pair padding, Activation act, const Tensor* residual = nullptr);
Tensor relu(const Tensor& input);
Tensor add(const Tensor& lhs, const Tensor& rhs);
Tensor mul(const Tensor& lhs, const Tensor& rhs);
Tensor max_pool2d(const Tensor& input, Pair kernel_size, Pair stride, Pair padding);
Tensor global_avg_pool(const Tensor& input);  // [N,C,H,W] -> [N,C]
// MatmulBackward::backward (rustorch-core/src/ops.rs:529-570) for
// out = lhs.matmul(rhs): {grad.matmul(rhs.t()), lhs.t().matmul(grad)}.
std::pair<Tensor, Tensor> matmul_backward(const Tensor& lhs, const Tensor& rhs,
                                          const Tensor& grad);
// Conv2dBackward::backward (rustorch-core/src/ops/conv.rs:648-736):
// {grad_input, grad_weight} of conv2d(input, weight, stride, padding).
std::pair<Tensor, Tensor> conv2d_backward(const Tensor& input, const Tensor& weight,
                                          const Tensor& grad, Pair stride, Pair padding);
}  // namespace ops

namespace nn {
struct Module {
  virtual ~Module() = default;
  virtual Tensor forward(const Tensor& input) const = 0;
  virtual std::vector<Tensor> parameters() const = 0;
};

// weight [out, in], bias [out]; forward = input.matmul(weight.t()) + bias
// (rustorch-nn/src/linear.rs:75-95), one kernel with the bias in the epilogue.
struct Linear : Module {
  Tensor weight;
  std::optional<Tensor> bias;
  // PyTorch-style U(-1/sqrt(in), 1/sqrt(in)) init from the seeded generator.
  Linear(size_t in_features, size_t out_features, uint64_t seed = 0, Device d = Device::cpu());
  Linear(Tensor w, std::optional<Tensor> b) : weight(std::move(w)), bias(std::move(b)) {}
  Tensor forward(const Tensor& input) const override;
  Tensor forward_fused(const Tensor& input, Activation act) const;
  std::vector<Tensor> parameters() const override;
};

// weight [out, in, kh, kw] (init 0.01 as the reference, rustorch-nn/src/conv.rs:29),
// bias [1, out, 1, 1] (zeros); forward = conv2d + broadcast bias, fused.
struct Conv2d : Module {
  Tensor weight;
  std::optional<Tensor> bias;
  Pair stride{1, 1}, padding{0, 0};
  Conv2d(size_t in_channels, size_t out_channels, Pair kernel_size, Pair stride, Pair padding,
         Device d = Device::cpu());
  Conv2d(Tensor w, std::optional<Tensor> b, Pair s, Pair p)
      : weight(std::move(w)), bias(std::move(b)), stride(s), padding(p) {}
  Tensor forward(const Tensor& input) const override;
  std::vector<Tensor> parameters() const override;
};
}  // namespace nn

namespace jit {
// NodeType (rustorch-core/src/jit.rs:7-21) plus Conv2dBiasRelu, the fused
// Conv2d -> Add(bias) -> Relu group this backend lowers to one kernel.
enum class Op { Input, Weight, Add, Mul, MatMul, Relu, Conv2d, Conv2dRelu, LinearRelu,
                Conv2dBiasRelu };

struct NodeType {
  Op op = Op::Input;
  size_t a = 0, b = 0, c = 0;  // operand node ids (Input: input index)
  Pair stride{1, 1}, padding{0, 0};
  Tensor weight;               // Weight nodes
  static NodeType Input(size_t index);
  static NodeType Weight(Tensor t);
  static NodeType Add(size_t lhs, size_t rhs);
  static NodeType Mul(size_t lhs, size_t rhs);
  static NodeType MatMul(size_t lhs, size_t rhs);
  static NodeType Relu(size_t x);
  static NodeType Conv2d(size_t input, size_t weight, Pair stride, Pair padding);
  static NodeType Conv2dRelu(size_t input, size_t weight, Pair stride, Pair padding);
  static NodeType LinearRelu(size_t input, size_t weight, size_t bias);
  static NodeType Conv2dBiasRelu(size_t input, size_t weight, size_t bias, Pair stride,
                                 Pair padding);
};

struct Node {
  NodeType op;
  std::vector<size_t> shape;
  size_t id = 0;
};

struct Graph {
  std::vector<Node> nodes;
  std::vector<size_t> inputs;
  std::vector<size_t> outputs;
  size_t add_node(NodeType op, std::vector<size_t> shape);
  size_t add_input(std::vector<size_t> shape);
  size_t add_weight(const Tensor& t);
};

struct Optimizer {
  // fuse_conv_relu (rustorch-core/src/jit.rs:85-209), then Conv2d -> Add(bias)
  // -> Relu chains on consecutive nodes into Conv2dBiasRelu.
  static void optimize(Graph& graph);
};

struct Executor {
  // Runs nodes in index order (rustorch-core/src/jit.rs:216-275); fused nodes
  // lower to one kernel each.
  static std::vector<Tensor> run(const Graph& graph, const std::vector<Tensor>& inputs);
};
}  // namespace jit

namespace vision {
// ResNet-18 inference forward composed from the ops above (the reference's
// rustorch-vision ResNet is an empty placeholder).  BatchNorm is folded into
// the conv weights/bias (gamma 1, beta 0, mean 0, var 1, eps 1e-5).
// Activations stay NHWC on the device between layers.
class ResNet18 {
 public:
  ResNet18(uint64_t seed, int device, int precision = RTB_PREC_3XTF32);
  ~ResNet18();
  ResNet18(const ResNet18&) = delete;
  ResNet18& operator=(const ResNet18&) = delete;
  // x: [B, 3, 224, 224] NCHW (CPU or CUDA); returns logits [B, 1000] on x's device.
  Tensor forward(const Tensor& x);
  // Device-pointer form (no allocation after the first call at a batch size).
  void forward_device(int64_t batch, const float* x_nchw, float* logits, void* stream);
  // Parameters in order: 20 conv weights [Co,Ci,kh,kw] each followed by its
  // bias [Co] (after BN folding), then fc.weight [1000,512], fc.bias [1000].
  size_t num_params() const;
  Tensor param(size_t i) const;
  int64_t flops_per_image() const;

 private:
  struct Impl;
  std::unique_ptr<Impl> impl_;
};
}  // namespace vision

}  // namespace rustorch
