// Implementation of the C++ mirror of RusTorch's operator interface
// (include/rustorch_b200.hpp) on top of the C ABI.  Every op is a call into
// the sm_100a kernels; CPU tensors are staged to the device and back.
#include <rustorch_b200.hpp>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <map>
#include <mutex>
#include <numeric>
#include <sstream>

namespace rustorch {

// ---------------------------------------------------------------- backend
namespace {

std::mutex g_ctx_mu;
rtb_ctx* g_ctx[64] = {nullptr};
int g_precision = RTB_PREC_3XTF32;

std::string last_error_text() {
  char buf[512];
  rtb_last_error(buf, sizeof buf);
  return buf;
}

void chk(int st, const char* what) {
  if (st != RTB_OK)
    throw Panic(std::string(what) + ": " + rtb_status_string(st) + ": " + last_error_text());
}

std::string shape_str(const std::vector<size_t>& s) {
  std::ostringstream o;
  o << "[";
  for (size_t i = 0; i < s.size(); ++i) o << (i ? ", " : "") << s[i];
  o << "]";
  return o.str();
}

size_t prod(const std::vector<size_t>& s) {
  return std::accumulate(s.begin(), s.end(), size_t(1), std::multiplies<size_t>());
}

std::vector<size_t> contiguous_strides(const std::vector<size_t>& shape) {
  std::vector<size_t> st(shape.size());
  size_t acc = 1;
  for (size_t i = shape.size(); i-- > 0;) {
    st[i] = acc;
    acc *= shape[i];
  }
  return st;
}

}  // namespace

rtb_ctx* context(int device) {
  if (device < 0 || device >= 64) throw Panic("device index out of range");
  std::lock_guard<std::mutex> lk(g_ctx_mu);
  if (!g_ctx[device]) chk(rtb_init(device, &g_ctx[device]), "rtb_init");
  return g_ctx[device];
}

void set_precision(int p) {
  if (p != RTB_PREC_3XTF32 && p != RTB_PREC_TF32) throw Panic("precision must be 3xTF32 or TF32");
  g_precision = p;
}
int precision() { return g_precision; }

void synchronize(int device) { chk(rtb_stream_synchronize(context(device), nullptr), "synchronize"); }

// ---------------------------------------------------------------- storage
struct Tensor::Storage {
  Device dev;
  size_t n = 0;
  std::vector<float> host;
  float* d = nullptr;
  explicit Storage(Device dv, size_t count) : dev(dv), n(count) {
    if (dev.is_cuda()) {
      void* p = nullptr;
      chk(rtb_malloc(context(dev.index), &p, std::max<size_t>(n, 1) * sizeof(float), nullptr),
          "device allocation");
      d = static_cast<float*>(p);
    } else {
      host.assign(n, 0.0f);
    }
  }
  ~Storage() {
    if (d) rtb_free(context(dev.index), d, nullptr);
  }
};

struct TensorAccess {
  static std::shared_ptr<Tensor::Storage>& storage(Tensor& t) { return t.storage_; }
  static const std::shared_ptr<Tensor::Storage>& storage(const Tensor& t) { return t.storage_; }
  static size_t offset(const Tensor& t) { return t.offset_; }
  static Tensor make(std::shared_ptr<Tensor::Storage> s, std::vector<size_t> shape,
                     std::vector<size_t> strides, size_t offset) {
    Tensor t;
    t.storage_ = std::move(s);
    t.shape_ = std::move(shape);
    t.strides_ = std::move(strides);
    t.offset_ = offset;
    return t;
  }
};

namespace {
Tensor make_contig(Device d, const std::vector<size_t>& shape) {
  auto s = std::make_shared<Tensor::Storage>(d, prod(shape));
  return TensorAccess::make(s, shape, contiguous_strides(shape), 0);
}
}  // namespace

Tensor Tensor::empty(const std::vector<size_t>& shape, Device d) { return make_contig(d, shape); }

Tensor Tensor::new_(const std::vector<float>& data, const std::vector<size_t>& shape) {
  const size_t size = prod(shape);
  if (data.size() != size)
    throw Panic("Data size " + std::to_string(data.size()) + " does not match shape " +
                shape_str(shape) + " (expected " + std::to_string(size) + ")");
  Tensor t = make_contig(Device::cpu(), shape);
  std::copy(data.begin(), data.end(), t.storage_->host.begin());
  return t;
}

Tensor Tensor::full(const std::vector<size_t>& shape, float v, Device d) {
  Tensor t = Tensor::new_(std::vector<float>(prod(shape), v), shape);
  return d.is_cuda() ? t.to(d) : t;
}
Tensor Tensor::zeros(const std::vector<size_t>& shape, Device d) { return full(shape, 0.f, d); }
Tensor Tensor::ones(const std::vector<size_t>& shape, Device d) { return full(shape, 1.f, d); }

Tensor Tensor::randn(const std::vector<size_t>& shape, uint64_t seed, uint64_t tid, float mean,
                     float sd, Device d) {
  Tensor t = make_contig(Device::cpu(), shape);
  chk(rtb_fill_normal_host(t.storage_->host.data(), (int64_t)t.numel(), seed, tid, mean, sd),
      "fill_normal");
  return d.is_cuda() ? t.to(d) : t;
}

Tensor Tensor::uniform(const std::vector<size_t>& shape, uint64_t seed, uint64_t tid, float lo,
                       float hi, Device d) {
  Tensor t = make_contig(Device::cpu(), shape);
  chk(rtb_fill_uniform_host(t.storage_->host.data(), (int64_t)t.numel(), seed, tid, lo, hi),
      "fill_uniform");
  return d.is_cuda() ? t.to(d) : t;
}

size_t Tensor::numel() const { return prod(shape_); }

bool Tensor::is_contiguous() const { return strides_ == contiguous_strides(shape_); }

Device Tensor::device() const { return storage_ ? storage_->dev : Device::cpu(); }

const float* Tensor::device_ptr() const {
  if (!storage_ || !storage_->dev.is_cuda()) throw Panic("device_ptr() on a CPU tensor");
  return storage_->d + offset_;
}
float* Tensor::device_ptr() {
  if (!storage_ || !storage_->dev.is_cuda()) throw Panic("device_ptr() on a CPU tensor");
  return storage_->d + offset_;
}

std::vector<float> Tensor::data() const {
  if (!storage_) return {};
  if (storage_->dev.is_cuda())
    throw Panic(
        "data() accessor only supported on CPU tensors. Use to_device() to move to CPU first.");
  std::vector<float> out(numel());
  if (is_contiguous()) {
    std::copy(storage_->host.begin() + offset_, storage_->host.begin() + offset_ + out.size(),
              out.begin());
    return out;
  }
  std::vector<size_t> idx(shape_.size(), 0);
  for (size_t i = 0; i < out.size(); ++i) {
    size_t off = offset_;
    for (size_t k = 0; k < idx.size(); ++k) off += idx[k] * strides_[k];
    out[i] = storage_->host[off];
    for (size_t k = idx.size(); k-- > 0;) {
      if (++idx[k] < shape_[k]) break;
      idx[k] = 0;
    }
  }
  return out;
}

namespace {
std::atomic<uint64_t> g_transfers{0};
}  // namespace

uint64_t transfer_count() { return g_transfers.load(); }

Tensor Tensor::to(Device d) const {
  if (!storage_) return *this;
  if (d == device()) return *this;
  if (d.is_cuda() != device().is_cuda()) g_transfers.fetch_add(1);
  Tensor src = contiguous();
  Tensor dst = make_contig(d, shape_);
  const size_t bytes = numel() * sizeof(float);
  if (d.is_cuda() && !src.device().is_cuda()) {
    chk(rtb_memcpy_h2d(context(d.index), dst.storage_->d,
                       src.storage_->host.data() + src.offset_, bytes, nullptr),
        "to(cuda)");
  } else if (!d.is_cuda() && src.device().is_cuda()) {
    chk(rtb_memcpy_d2h(context(src.device().index), dst.storage_->host.data(),
                       src.storage_->d + src.offset_, bytes, nullptr),
        "to(cpu)");
    synchronize(src.device().index);
  } else {  // device to device
    Tensor tmp = src.to(Device::cpu());
    return tmp.to(d);
  }
  return dst;
}

Tensor Tensor::t() const {
  if (dim() != 2) throw Panic("t() expects a 2-D tensor");
  return permute({1, 0});
}

Tensor Tensor::permute(const std::vector<size_t>& dims) const {
  if (dims.size() != dim()) throw Panic("Invalid permutation " + shape_str(dims));
  std::vector<bool> seen(dims.size(), false);
  std::vector<size_t> sh(dims.size()), st(dims.size());
  for (size_t i = 0; i < dims.size(); ++i) {
    if (dims[i] >= dims.size() || seen[dims[i]]) throw Panic("Invalid permutation " + shape_str(dims));
    seen[dims[i]] = true;
    sh[i] = shape_[dims[i]];
    st[i] = strides_[dims[i]];
  }
  return TensorAccess::make(storage_, sh, st, offset_);
}

Tensor Tensor::reshape(const std::vector<size_t>& shape) const {
  if (prod(shape) != numel()) throw Panic("reshape: element count differs");
  Tensor c = contiguous();
  return TensorAccess::make(c.storage_, shape, contiguous_strides(shape), c.offset_);
}

Tensor Tensor::contiguous() const {
  if (!storage_ || is_contiguous()) return *this;
  if (!storage_->dev.is_cuda()) return Tensor::new_(data(), shape_);
  // Device strided copy: y = x + 0 with a broadcast zero (strided gather).
  Tensor out = make_contig(storage_->dev, shape_);
  Tensor zero = Tensor::zeros({1}, storage_->dev);
  std::vector<int64_t> sh(shape_.begin(), shape_.end()), sa(strides_.begin(), strides_.end()),
      sb(shape_.size(), 0);
  if (sh.empty()) {
    sh = {1};
    sa = {0};
    sb = {0};
  }
  chk(rtb_elementwise_broadcast(context(storage_->dev.index), 0, (int)sh.size(), sh.data(),
                                device_ptr(), sa.data(), zero.device_ptr(), sb.data(),
                                out.device_ptr(), nullptr),
      "contiguous");
  return out;
}

Tensor Tensor::matmul(const Tensor& rhs) const { return ops::matmul(*this, rhs); }
Tensor Tensor::conv2d(const Tensor& w, Pair stride, Pair padding) const {
  return ops::conv2d(*this, w, stride, padding);
}
Tensor Tensor::relu() const { return ops::relu(*this); }
Tensor Tensor::add(const Tensor& rhs) const { return ops::add(*this, rhs); }
Tensor Tensor::mul(const Tensor& rhs) const { return ops::mul(*this, rhs); }

// ---------------------------------------------------------------- ops
namespace {

// The device all operands share; CPU operands are staged to device 0.
struct Placement {
  bool host = false;  // every operand was on the CPU
  int device = 0;
};

Placement place(std::initializer_list<const Tensor*> ts) {
  Placement p;
  bool any_cpu = false, any_cuda = false;
  int dev = -1;
  for (const Tensor* t : ts) {
    if (!t || !t->defined()) continue;
    if (t->device().is_cuda()) {
      any_cuda = true;
      if (dev >= 0 && dev != t->device().index)
        throw Panic("tensors are on different CUDA devices");
      dev = t->device().index;
    } else {
      any_cpu = true;
    }
  }
  if (any_cpu && any_cuda) throw Panic("tensors are on different devices (CPU and CUDA)");
  p.host = !any_cuda;
  p.device = dev < 0 ? 0 : dev;
  return p;
}

Tensor on(const Tensor& t, const Placement& p) {
  return t.device().is_cuda() ? t : t.to(Device::cuda(p.device));
}

Tensor finish(Tensor out, const Placement& p) { return p.host ? out.to_cpu() : out; }

// (ld, trans) describing a 2-D CUDA view for rtb_sgemm; copies only when
// neither dimension is unit-stride.
Tensor gemm_operand(const Tensor& t, int64_t& ld, int& trans) {
  const auto& st = t.strides();
  const auto& sh = t.shape();
  if (st[1] == 1 && st[0] >= std::max<size_t>(sh[1], 1)) {
    ld = (int64_t)st[0];
    trans = 0;
    return t;
  }
  if (st[0] == 1 && st[1] >= std::max<size_t>(sh[0], 1)) {
    ld = (int64_t)st[1];
    trans = 1;
    return t;
  }
  Tensor c = t.contiguous();
  ld = (int64_t)sh[1];
  trans = 0;
  return c;
}

Tensor broadcast_op(const Tensor& lhs, const Tensor& rhs, int op) {
  Placement p = place({&lhs, &rhs});
  // broadcast_shapes (rustorch-core/src/broadcast.rs): right-aligned, 1 stretches.
  const size_t nd = std::max(lhs.dim(), rhs.dim());
  std::vector<size_t> out(nd);
  std::vector<int64_t> sa(nd, 0), sb(nd, 0);
  for (size_t i = 0; i < nd; ++i) {
    const size_t ia = i + lhs.dim() >= nd ? i + lhs.dim() - nd : SIZE_MAX;
    const size_t ib = i + rhs.dim() >= nd ? i + rhs.dim() - nd : SIZE_MAX;
    const size_t da = ia == SIZE_MAX ? 1 : lhs.shape()[ia];
    const size_t db = ib == SIZE_MAX ? 1 : rhs.shape()[ib];
    if (da != db && da != 1 && db != 1)
      throw Panic("Shapes not broadcastable: " + shape_str(lhs.shape()) + " vs " +
                  shape_str(rhs.shape()));
    out[i] = std::max(da, db);
    sa[i] = (ia == SIZE_MAX || da == 1) ? 0 : (int64_t)lhs.strides()[ia];
    sb[i] = (ib == SIZE_MAX || db == 1) ? 0 : (int64_t)rhs.strides()[ib];
  }
  Tensor a = on(lhs, p), b = on(rhs, p);
  Tensor y = make_contig(Device::cuda(p.device), out);
  std::vector<int64_t> sh(out.begin(), out.end());
  if (sh.empty()) {
    sh = {1};
    sa = {0};
    sb = {0};
  }
  chk(rtb_elementwise_broadcast(context(p.device), op, (int)sh.size(), sh.data(), a.device_ptr(),
                                sa.data(), b.device_ptr(), sb.data(), y.device_ptr(), nullptr),
      op == 0 ? "add" : "mul");
  return finish(y, p);
}

}  // namespace

namespace ops {

Tensor matmul_fused(const Tensor& lhs, const Tensor& rhs, const Tensor* bias, Activation act) {
  if (lhs.dim() != 2 || rhs.dim() != 2) throw Panic("Matmul only supports 2D");
  const size_t m = lhs.shape()[0], k = lhs.shape()[1], k2 = rhs.shape()[0], n = rhs.shape()[1];
  if (k != k2) throw Panic("Matmul dimension mismatch");
  if (bias && (bias->numel() != n)) throw Panic("matmul_fused: bias must have N elements");
  Placement p = place({&lhs, &rhs, bias});
  Tensor a = on(lhs, p), b = on(rhs, p);
  Tensor bz = bias ? on(*bias, p).contiguous() : Tensor();
  Tensor y = make_contig(Device::cuda(p.device), {m, n});
  if (m && n) {
    int64_t lda, ldb;
    int ta, tb;
    Tensor a2 = k ? gemm_operand(a, lda, ta) : a, b2 = k ? gemm_operand(b, ldb, tb) : b;
    if (!k) {
      lda = 1;
      ldb = (int64_t)n;
      ta = tb = 0;
    }
    chk(rtb_sgemm(context(p.device), (int64_t)m, (int64_t)n, (int64_t)k,
                  k ? a2.device_ptr() : nullptr, lda, ta, k ? b2.device_ptr() : nullptr, ldb, tb,
                  bias ? bz.device_ptr() : nullptr, static_cast<int>(act), y.device_ptr(),
                  (int64_t)n, g_precision, nullptr),
        "matmul");
  }
  return finish(y, p);
}

Tensor matmul_bias_norm_activation(const Tensor& lhs, const Tensor& rhs, const Tensor* bias,
                                   const Tensor* norm_weight, const Tensor* norm_bias, float eps,
                                   Activation act) {
  if (lhs.dim() != 2 || rhs.dim() != 2) throw Panic("Matmul only supports 2D");
  const size_t m = lhs.shape()[0], k = lhs.shape()[1], k2 = rhs.shape()[0], n = rhs.shape()[1];
  if (k != k2) throw Panic("Matmul dimension mismatch");
  for (const Tensor* t : {bias, norm_weight, norm_bias})
    if (t && t->numel() != n)
      throw Panic("LayerNorm: Input shape does not match normalized shape");
  Placement p = place({&lhs, &rhs, bias, norm_weight, norm_bias});
  Tensor a = on(lhs, p), b = on(rhs, p);
  Tensor bz = bias ? on(*bias, p).contiguous() : Tensor();
  Tensor gz = norm_weight ? on(*norm_weight, p).contiguous() : Tensor();
  Tensor nz = norm_bias ? on(*norm_bias, p).contiguous() : Tensor();
  Tensor y = make_contig(Device::cuda(p.device), {m, n});
  if (m && n) {
    int64_t lda = 1, ldb = (int64_t)n;
    int ta = 0, tb = 0;
    Tensor a2 = k ? gemm_operand(a, lda, ta) : a, b2 = k ? gemm_operand(b, ldb, tb) : b;
    chk(rtb_matmul_bias_norm_act(context(p.device), (int64_t)m, (int64_t)n, (int64_t)k,
                                 k ? a2.device_ptr() : nullptr, lda, ta,
                                 k ? b2.device_ptr() : nullptr, ldb, tb,
                                 bias ? bz.device_ptr() : nullptr,
                                 norm_weight ? gz.device_ptr() : nullptr,
                                 norm_bias ? nz.device_ptr() : nullptr, eps,
                                 static_cast<int>(act), y.device_ptr(), (int64_t)n, g_precision,
                                 nullptr),
        "matmul_bias_norm_activation");
  }
  return finish(y, p);
}

Tensor matmul(const Tensor& lhs, const Tensor& rhs) {
  return matmul_fused(lhs, rhs, nullptr, Activation::None);
}

Tensor conv2d_fused(const Tensor& input, const Tensor& weight, const Tensor* bias, Pair stride,
                    Pair padding, Activation act, const Tensor* residual) {
  if (input.dim() != 4 || weight.dim() != 4) throw Panic("Conv2d requires 4D tensors");
  const auto& is = input.shape();
  const auto& ws = weight.shape();
  if (ws[1] != is[1])
    throw Panic("Weight input channels " + std::to_string(ws[1]) + " must match input channels " +
                std::to_string(is[1]));
  const size_t N = is[0], C = is[1], H = is[2], W = is[3], Co = ws[0], kh = ws[2], kw = ws[3];
  if (H + 2 * padding.first < kh || W + 2 * padding.second < kw)
    throw Panic("Conv2d: kernel larger than padded input");
  const size_t Ho = (H + 2 * padding.first - kh) / stride.first + 1;
  const size_t Wo = (W + 2 * padding.second - kw) / stride.second + 1;
  if (bias && bias->numel() != Co) throw Panic("conv2d: bias must have out_channels elements");
  if (residual && residual->shape() != std::vector<size_t>{N, Co, Ho, Wo})
    throw Panic("conv2d: residual shape must equal the output shape");
  Placement p = place({&input, &weight, bias, residual});
  Tensor x = on(input, p).contiguous(), w = on(weight, p).contiguous();
  Tensor b = bias ? on(*bias, p).contiguous() : Tensor();
  Tensor r = residual ? on(*residual, p).contiguous() : Tensor();
  Tensor y = make_contig(Device::cuda(p.device), {N, Co, Ho, Wo});
  chk(rtb_conv2d_fwd(context(p.device), (int64_t)N, (int64_t)C, (int64_t)H, (int64_t)W,
                     (int64_t)Co, (int64_t)kh, (int64_t)kw, (int64_t)stride.first,
                     (int64_t)stride.second, (int64_t)padding.first, (int64_t)padding.second,
                     x.device_ptr(), RTB_LAYOUT_NCHW, w.device_ptr(),
                     bias ? b.device_ptr() : nullptr, residual ? r.device_ptr() : nullptr,
                     static_cast<int>(act), y.device_ptr(), RTB_LAYOUT_NCHW, g_precision,
                     nullptr),
      "conv2d");
  return finish(y, p);
}

Tensor conv2d(const Tensor& input, const Tensor& weight, Pair stride, Pair padding) {
  return conv2d_fused(input, weight, nullptr, stride, padding, Activation::None, nullptr);
}

Tensor relu(const Tensor& input) {
  Placement p = place({&input});
  Tensor x = on(input, p).contiguous();
  Tensor y = make_contig(Device::cuda(p.device), input.shape());
  chk(rtb_relu(context(p.device), (int64_t)x.numel(), x.device_ptr(), y.device_ptr(), nullptr),
      "relu");
  return finish(y, p);
}

Tensor add(const Tensor& lhs, const Tensor& rhs) { return broadcast_op(lhs, rhs, 0); }
Tensor mul(const Tensor& lhs, const Tensor& rhs) { return broadcast_op(lhs, rhs, 1); }

Tensor max_pool2d(const Tensor& input, Pair k, Pair s, Pair pd) {
  if (input.dim() != 4) throw Panic("MaxPool2d requires 4D tensor (N, C, H, W)");
  Placement p = place({&input});
  Tensor x = on(input, p).contiguous();
  const auto& sh = input.shape();
  const size_t Ho = (sh[2] + 2 * pd.first - k.first) / s.first + 1;
  const size_t Wo = (sh[3] + 2 * pd.second - k.second) / s.second + 1;
  Tensor y = make_contig(Device::cuda(p.device), {sh[0], sh[1], Ho, Wo});
  chk(rtb_max_pool2d(context(p.device), (int64_t)sh[0], (int64_t)sh[1], (int64_t)sh[2],
                     (int64_t)sh[3], (int64_t)k.first, (int64_t)k.second, (int64_t)s.first,
                     (int64_t)s.second, (int64_t)pd.first, (int64_t)pd.second, x.device_ptr(),
                     y.device_ptr(), RTB_LAYOUT_NCHW, nullptr),
      "max_pool2d");
  return finish(y, p);
}

std::pair<Tensor, Tensor> matmul_backward(const Tensor& lhs, const Tensor& rhs,
                                          const Tensor& grad) {
  if (lhs.dim() != 2 || rhs.dim() != 2 || grad.dim() != 2) throw Panic("Matmul only supports 2D");
  const size_t m = lhs.shape()[0], k = lhs.shape()[1], n = rhs.shape()[1];
  if (rhs.shape()[0] != k || grad.shape()[0] != m || grad.shape()[1] != n)
    throw Panic("Matmul dimension mismatch");
  Placement p = place({&lhs, &rhs, &grad});
  Tensor a = on(lhs, p).contiguous(), b = on(rhs, p).contiguous(), g = on(grad, p).contiguous();
  Tensor da = make_contig(Device::cuda(p.device), {m, k});
  Tensor db = make_contig(Device::cuda(p.device), {k, n});
  chk(rtb_matmul_backward(context(p.device), (int64_t)m, (int64_t)n, (int64_t)k, a.device_ptr(),
                          b.device_ptr(), g.device_ptr(), da.device_ptr(), db.device_ptr(), 0,
                          g_precision, nullptr),
      "matmul_backward");
  return {finish(da, p), finish(db, p)};
}

std::pair<Tensor, Tensor> conv2d_backward(const Tensor& input, const Tensor& weight,
                                          const Tensor& grad, Pair stride, Pair padding) {
  if (input.dim() != 4 || weight.dim() != 4 || grad.dim() != 4)
    throw Panic("Conv2d requires 4D tensors");
  const auto& is = input.shape();
  const auto& ws = weight.shape();
  Placement p = place({&input, &weight, &grad});
  Tensor x = on(input, p).contiguous(), w = on(weight, p).contiguous();
  Tensor g = on(grad, p).contiguous();
  Tensor dx = make_contig(Device::cuda(p.device), is);
  Tensor dw = make_contig(Device::cuda(p.device), ws);
  chk(rtb_conv2d_backward(context(p.device), (int64_t)is[0], (int64_t)is[1], (int64_t)is[2],
                          (int64_t)is[3], (int64_t)ws[0], (int64_t)ws[2], (int64_t)ws[3],
                          (int64_t)stride.first, (int64_t)stride.second, (int64_t)padding.first,
                          (int64_t)padding.second, x.device_ptr(), w.device_ptr(), g.device_ptr(),
                          dx.device_ptr(), dw.device_ptr(), 0, g_precision, nullptr),
      "conv2d_backward");
  return {finish(dx, p), finish(dw, p)};
}

Tensor global_avg_pool(const Tensor& input) {
  if (input.dim() != 4) throw Panic("global_avg_pool requires 4D tensor (N, C, H, W)");
  Placement p = place({&input});
  Tensor x = on(input, p).contiguous();
  const auto& sh = input.shape();
  Tensor y = make_contig(Device::cuda(p.device), {sh[0], sh[1]});
  chk(rtb_global_avg_pool(context(p.device), (int64_t)sh[0], (int64_t)sh[1], (int64_t)sh[2],
                          (int64_t)sh[3], x.device_ptr(), y.device_ptr(), RTB_LAYOUT_NCHW,
                          nullptr),
      "global_avg_pool");
  return finish(y, p);
}

}  // namespace ops

// ---------------------------------------------------------------- nn
namespace nn {

Linear::Linear(size_t in, size_t out, uint64_t seed, Device d) {
  const float k = 1.0f / std::sqrt((float)in);
  weight = Tensor::uniform({out, in}, seed, 0, -k, k, d);
  bias = Tensor::uniform({out}, seed, 1, -k, k, d);
}

Tensor Linear::forward(const Tensor& input) const { return forward_fused(input, Activation::None); }

Tensor Linear::forward_fused(const Tensor& input, Activation act) const {
  // y = input.matmul(weight.t()) + bias: weight.t() is a K-major view, the
  // bias and activation run in the GEMM epilogue.
  return ops::matmul_fused(input, weight.t(), bias ? &*bias : nullptr, act);
}

std::vector<Tensor> Linear::parameters() const {
  std::vector<Tensor> p{weight};
  if (bias) p.push_back(*bias);
  return p;
}

Conv2d::Conv2d(size_t in, size_t out, Pair k, Pair s, Pair p, Device d) : stride(s), padding(p) {
  weight = Tensor::full({out, in, k.first, k.second}, 0.01f, d);
  bias = Tensor::zeros({1, out, 1, 1}, d);
}

Tensor Conv2d::forward(const Tensor& input) const {
  return ops::conv2d_fused(input, weight, bias ? &*bias : nullptr, stride, padding,
                           Activation::None, nullptr);
}

std::vector<Tensor> Conv2d::parameters() const {
  std::vector<Tensor> p{weight};
  if (bias) p.push_back(*bias);
  return p;
}

}  // namespace nn

// ---------------------------------------------------------------- jit
namespace jit {

NodeType NodeType::Input(size_t i) { NodeType n; n.op = Op::Input; n.a = i; return n; }
NodeType NodeType::Weight(Tensor t) { NodeType n; n.op = Op::Weight; n.weight = std::move(t); return n; }
NodeType NodeType::Add(size_t a, size_t b) { NodeType n; n.op = Op::Add; n.a = a; n.b = b; return n; }
NodeType NodeType::Mul(size_t a, size_t b) { NodeType n; n.op = Op::Mul; n.a = a; n.b = b; return n; }
NodeType NodeType::MatMul(size_t a, size_t b) { NodeType n; n.op = Op::MatMul; n.a = a; n.b = b; return n; }
NodeType NodeType::Relu(size_t a) { NodeType n; n.op = Op::Relu; n.a = a; return n; }
NodeType NodeType::Conv2d(size_t i, size_t w, Pair s, Pair p) {
  NodeType n; n.op = Op::Conv2d; n.a = i; n.b = w; n.stride = s; n.padding = p; return n;
}
NodeType NodeType::Conv2dRelu(size_t i, size_t w, Pair s, Pair p) {
  NodeType n; n.op = Op::Conv2dRelu; n.a = i; n.b = w; n.stride = s; n.padding = p; return n;
}
NodeType NodeType::LinearRelu(size_t i, size_t w, size_t b) {
  NodeType n; n.op = Op::LinearRelu; n.a = i; n.b = w; n.c = b; return n;
}
NodeType NodeType::Conv2dBiasRelu(size_t i, size_t w, size_t b, Pair s, Pair p) {
  NodeType n; n.op = Op::Conv2dBiasRelu; n.a = i; n.b = w; n.c = b; n.stride = s; n.padding = p;
  return n;
}

size_t Graph::add_node(NodeType op, std::vector<size_t> shape) {
  const size_t id = nodes.size();
  nodes.push_back(Node{std::move(op), std::move(shape), id});
  return id;
}
size_t Graph::add_input(std::vector<size_t> shape) {
  const size_t id = add_node(NodeType::Input(inputs.size()), std::move(shape));
  inputs.push_back(id);
  return id;
}
size_t Graph::add_weight(const Tensor& t) { return add_node(NodeType::Weight(t), t.shape()); }

namespace {
size_t remap(const std::map<size_t, size_t>& m, size_t i) {
  auto it = m.find(i);
  return it == m.end() ? i : it->second;
}

// Rebuild pass over index order: Conv2d(i) followed by Relu(i) at i+1 becomes
// Conv2dRelu (jit.rs:85-209); with bias fusion also Conv2d(i) -> Add(i, b) at
// i+1 -> Relu(i+1) at i+2 becomes Conv2dBiasRelu.
void fuse(Graph& g) {
  std::vector<Node> out;
  std::map<size_t, size_t> map;
  const size_t n = g.nodes.size();
  std::vector<bool> consumed(n, false);
  for (size_t i = 0; i < n; ++i) {
    if (consumed[i]) continue;
    const Node& node = g.nodes[i];
    if (node.op.op == Op::Conv2d) {
      const NodeType& c = node.op;
      if (i + 2 < n && g.nodes[i + 1].op.op == Op::Add && g.nodes[i + 1].op.a == i &&
          g.nodes[i + 2].op.op == Op::Relu && g.nodes[i + 2].op.a == i + 1) {
        const size_t id = out.size();
        map[i + 2] = id;
        out.push_back(Node{NodeType::Conv2dBiasRelu(remap(map, c.a), remap(map, c.b),
                                                    remap(map, g.nodes[i + 1].op.b), c.stride,
                                                    c.padding),
                           g.nodes[i + 2].shape, id});
        consumed[i + 1] = consumed[i + 2] = true;
        continue;
      }
      if (i + 1 < n && g.nodes[i + 1].op.op == Op::Relu && g.nodes[i + 1].op.a == i) {
        const size_t id = out.size();
        map[i + 1] = id;
        out.push_back(Node{NodeType::Conv2dRelu(remap(map, c.a), remap(map, c.b), c.stride,
                                                c.padding),
                           g.nodes[i + 1].shape, id});
        consumed[i + 1] = true;
        continue;
      }
    }
    const size_t id = out.size();
    map[i] = id;
    NodeType op = node.op;
    switch (op.op) {
      case Op::Add: case Op::Mul: case Op::MatMul:
        op.a = remap(map, op.a); op.b = remap(map, op.b); break;
      case Op::Relu: op.a = remap(map, op.a); break;
      case Op::Conv2d: case Op::Conv2dRelu:
        op.a = remap(map, op.a); op.b = remap(map, op.b); break;
      case Op::LinearRelu: case Op::Conv2dBiasRelu:
        op.a = remap(map, op.a); op.b = remap(map, op.b); op.c = remap(map, op.c); break;
      default: break;
    }
    out.push_back(Node{op, node.shape, id});
  }
  g.nodes = std::move(out);
  for (auto& o : g.outputs) o = remap(map, o);
  for (auto& i : g.inputs) i = remap(map, i);
}
}  // namespace

void Optimizer::optimize(Graph& graph) { fuse(graph); }

// Device-resident execution: CPU inputs and weights move to the device once,
// every node runs on device tensors (no per-node host round trip), and the
// outputs come back to the CPU at the end (jit.rs:216 runs nodes in index
// order on whatever the inputs are; results are returned where they were).
std::vector<Tensor> Executor::run(const Graph& graph, const std::vector<Tensor>& inputs) {
  std::map<size_t, Tensor> values;
  bool host = false;
  int dev = -1;
  for (size_t i = 0; i < graph.inputs.size() && i < inputs.size(); ++i) {
    if (!inputs[i].defined()) continue;
    if (inputs[i].device().is_cuda()) {
      if (dev < 0) dev = inputs[i].device().index;
    } else {
      host = true;
    }
  }
  if (dev < 0) dev = 0;
  const Device on_dev = Device::cuda(dev);
  for (size_t i = 0; i < graph.inputs.size(); ++i) {
    if (i >= inputs.size()) throw Panic("Executor::run: missing input");
    values[graph.inputs[i]] = inputs[i].defined() ? inputs[i].to(on_dev) : inputs[i];
  }
  auto get = [&](size_t id) -> const Tensor& {
    auto it = values.find(id);
    if (it == values.end()) throw Panic("Executor::run: node used before it was computed");
    return it->second;
  };
  for (const Node& node : graph.nodes) {
    if (values.count(node.id)) continue;
    const NodeType& op = node.op;
    Tensor v;
    switch (op.op) {
      case Op::Input: throw Panic("Input should be loaded");
      case Op::Weight: v = op.weight.defined() ? op.weight.to(on_dev) : op.weight; break;
      case Op::Add: v = get(op.a).add(get(op.b)); break;
      case Op::Mul: v = get(op.a).mul(get(op.b)); break;
      case Op::MatMul: v = get(op.a).matmul(get(op.b)); break;
      case Op::Relu: v = get(op.a).relu(); break;
      case Op::Conv2d: v = get(op.a).conv2d(get(op.b), op.stride, op.padding); break;
      case Op::Conv2dRelu:
        v = ops::conv2d_fused(get(op.a), get(op.b), nullptr, op.stride, op.padding,
                              Activation::ReLU);
        break;
      case Op::Conv2dBiasRelu: {
        const Tensor& b = get(op.c);
        v = ops::conv2d_fused(get(op.a), get(op.b), &b, op.stride, op.padding, Activation::ReLU);
        break;
      }
      case Op::LinearRelu: {
        const Tensor& b = get(op.c);
        v = ops::matmul_fused(get(op.a), get(op.b).t(), &b, Activation::ReLU);
        break;
      }
    }
    values[node.id] = v;
  }
  std::vector<Tensor> out;
  for (size_t id : graph.outputs) out.push_back(host ? get(id).to_cpu() : get(id));
  return out;
}

}  // namespace jit

// ---------------------------------------------------------------- vision
namespace vision {

namespace {
struct ConvSpec {
  size_t ci, co, k, s, p;
};
}  // namespace

struct ResNet18::Impl {
  int device = 0;
  int prec = RTB_PREC_3XTF32;
  std::vector<ConvSpec> specs;
  std::vector<Tensor> w, b;    // folded conv weights [Co,Ci,k,k] / bias [Co] (device)
  std::vector<Tensor> wp;      // prepacked weights [Co, k*k*Cp] (device)
  std::vector<Tensor> wlo;     // their 3xTF32 low parts, same layout (device)
  Tensor fc_w, fc_b;           // [1000,512], [1000] (device)
  int64_t cap_batch = 0;
  Tensor bufA, bufB, bufC, bufD, pooled;  // NHWC activation buffers
};

ResNet18::ResNet18(uint64_t seed, int device, int prec) : impl_(new Impl) {
  auto& I = *impl_;
  I.device = device;
  I.prec = prec;
  const Device d = Device::cuda(device);
  // conv table: stem, then per stage [conv_a, conv_b, (downsample)], 2 blocks each.
  I.specs.push_back({3, 64, 7, 2, 3});
  const size_t widths[4] = {64, 128, 256, 512};
  size_t cin = 64;
  for (int st = 0; st < 4; ++st) {
    const size_t co = widths[st];
    for (int blk = 0; blk < 2; ++blk) {
      const size_t s = (st > 0 && blk == 0) ? 2 : 1;
      I.specs.push_back({cin, co, 3, s, 1});
      I.specs.push_back({co, co, 3, 1, 1});
      if (st > 0 && blk == 0) I.specs.push_back({cin, co, 1, 2, 0});
      cin = co;
    }
  }
  const float bn_scale = 1.0f / std::sqrt(1.0f + 1e-5f);
  for (size_t i = 0; i < I.specs.size(); ++i) {
    const auto& c = I.specs[i];
    const float sd = std::sqrt(2.0f / (float)(c.ci * c.k * c.k)) * bn_scale;  // Kaiming-normal, BN folded
    I.w.push_back(Tensor::randn({c.co, c.ci, c.k, c.k}, seed, i, 0.0f, sd, d));
    I.b.push_back(Tensor::zeros({c.co}, d));  // beta - mean * scale = 0
    const int64_t n = rtb_conv2d_packed_weight_size((int64_t)c.co, (int64_t)c.ci, (int64_t)c.k,
                                                    (int64_t)c.k);
    Tensor packed = Tensor::empty({(size_t)n}, d);
    Tensor lo = Tensor::empty({(size_t)n}, d);
    chk(rtb_conv2d_prepack_weight_lo(context(device), (int64_t)c.co, (int64_t)c.ci, (int64_t)c.k,
                                     (int64_t)c.k, I.w.back().device_ptr(), packed.device_ptr(),
                                     lo.device_ptr(), nullptr),
        "prepack");
    I.wp.push_back(packed);
    I.wlo.push_back(lo);
  }
  const float k = 1.0f / std::sqrt(512.0f);
  I.fc_w = Tensor::uniform({1000, 512}, seed, 100, -k, k, d);
  I.fc_b = Tensor::uniform({1000}, seed, 101, -k, k, d);
}

ResNet18::~ResNet18() = default;

size_t ResNet18::num_params() const { return impl_->w.size() * 2 + 2; }

Tensor ResNet18::param(size_t i) const {
  const auto& I = *impl_;
  if (i < I.w.size() * 2) return (i % 2 == 0) ? I.w[i / 2] : I.b[i / 2];
  if (i == I.w.size() * 2) return I.fc_w;
  if (i == I.w.size() * 2 + 1) return I.fc_b;
  throw Panic("ResNet18::param index out of range");
}

int64_t ResNet18::flops_per_image() const {
  // 2 * MACs of every conv and the FC, walking the network as forward_device does.
  const auto& S = impl_->specs;
  auto conv_flops = [](const ConvSpec& c, int64_t ho) {
    return 2 * ho * ho * (int64_t)c.co * (int64_t)(c.ci * c.k * c.k);
  };
  auto out = [](int64_t h, const ConvSpec& c) {
    return (h + 2 * (int64_t)c.p - (int64_t)c.k) / (int64_t)c.s + 1;
  };
  int64_t h = out(224, S[0]);
  int64_t f = conv_flops(S[0], h);
  h = (h + 2 - 3) / 2 + 1;  // max pool 3x3 s2 p1
  size_t i = 1;
  for (int st = 0; st < 4; ++st)
    for (int blk = 0; blk < 2; ++blk) {
      const bool down = (st > 0 && blk == 0);
      const int64_t ho = out(h, S[i]);
      f += conv_flops(S[i], ho) + conv_flops(S[i + 1], ho);
      if (down) f += conv_flops(S[i + 2], ho);
      i += down ? 3 : 2;
      h = ho;
    }
  return f + 2 * 512 * 1000;
}

void ResNet18::forward_device(int64_t B, const float* x_nchw, float* logits, void* stream) {
  auto& I = *impl_;
  rtb_ctx* ctx = context(I.device);
  const Device d = Device::cuda(I.device);
  if (B > I.cap_batch) {
    const size_t b = (size_t)B;
    const size_t big = b * 112 * 112 * 64;  // largest activation (stem output)
    I.bufA = Tensor::empty({big}, d);
    I.bufB = Tensor::empty({big}, d);
    I.bufC = Tensor::empty({big}, d);
    I.bufD = Tensor::empty({big}, d);
    I.pooled = Tensor::empty({b * 512}, d);
    I.cap_batch = B;
  }
  auto conv = [&](size_t i, const float* x, int64_t H, int64_t W, float* y, const float* res,
                  bool relu) {
    const auto& c = I.specs[i];
    chk(rtb_conv2d_fwd_packed_lo(ctx, B, (int64_t)c.ci, H, W, (int64_t)c.co, (int64_t)c.k,
                                 (int64_t)c.k, (int64_t)c.s, (int64_t)c.s, (int64_t)c.p,
                                 (int64_t)c.p, x, I.wp[i].device_ptr(), I.wlo[i].device_ptr(),
                                 I.b[i].device_ptr(), res, relu ? RTB_ACT_RELU : RTB_ACT_NONE, y,
                                 RTB_LAYOUT_NHWC, I.prec, stream),
        "resnet conv");
    return (H + 2 * (int64_t)c.p - (int64_t)c.k) / (int64_t)c.s + 1;
  };
  // stem straight from the NCHW input (the conv's prologue writes the stride-2
  // space-to-depth layout in 3xTF32 mode, NHWC otherwise)
  {
    const auto& c = I.specs[0];
    chk(rtb_conv2d_fwd(ctx, B, (int64_t)c.ci, 224, 224, (int64_t)c.co, (int64_t)c.k, (int64_t)c.k,
                       (int64_t)c.s, (int64_t)c.s, (int64_t)c.p, (int64_t)c.p, x_nchw,
                       RTB_LAYOUT_NCHW, I.w[0].device_ptr(), I.b[0].device_ptr(), nullptr,
                       RTB_ACT_RELU, I.bufA.device_ptr(), RTB_LAYOUT_NHWC, I.prec, stream),
        "resnet stem");
  }
  int64_t h = (224 + 2 * 3 - 7) / 2 + 1;  // 112
  chk(rtb_max_pool2d(ctx, B, 64, h, h, 3, 3, 2, 2, 1, 1, I.bufA.device_ptr(), I.bufB.device_ptr(),
                     RTB_LAYOUT_NHWC, stream),
      "resnet maxpool");
  h = (h + 2 - 3) / 2 + 1;  // 56
  float* cur = I.bufB.device_ptr();
  float* t1 = I.bufA.device_ptr();
  float* t2 = I.bufC.device_ptr();
  float* t3 = I.bufD.device_ptr();
  size_t i = 1;
  for (int st = 0; st < 4; ++st) {
    for (int blk = 0; blk < 2; ++blk) {
      const bool down = (st > 0 && blk == 0);
      const int64_t ho = conv(i, cur, h, h, t1, nullptr, true);  // conv_a + bias + relu
      const float* identity = cur;
      if (down) {
        conv(i + 2, cur, h, h, t3, nullptr, false);  // 1x1 s2 downsample + bias
        identity = t3;
      }
      conv(i + 1, t1, ho, ho, t2, identity, true);  // conv_b + bias + residual + relu
      i += down ? 3 : 2;
      std::swap(cur, t2);
      h = ho;
    }
  }
  chk(rtb_global_avg_pool(ctx, B, 512, h, h, cur, I.pooled.device_ptr(), RTB_LAYOUT_NHWC, stream),
      "resnet avgpool");
  chk(rtb_sgemm(ctx, B, 1000, 512, I.pooled.device_ptr(), 512, 0, I.fc_w.device_ptr(), 512, 1,
                I.fc_b.device_ptr(), RTB_ACT_NONE, logits, 1000, I.prec, stream),
      "resnet fc");
}

Tensor ResNet18::forward(const Tensor& x) {
  if (x.dim() != 4 || x.shape()[1] != 3 || x.shape()[2] != 224 || x.shape()[3] != 224)
    throw Panic("ResNet18 expects [B, 3, 224, 224]");
  const bool host = !x.device().is_cuda();
  Tensor xd = x.to(Device::cuda(impl_->device)).contiguous();
  Tensor y = Tensor::empty({x.shape()[0], 1000}, Device::cuda(impl_->device));
  forward_device((int64_t)x.shape()[0], xd.device_ptr(), y.device_ptr(), nullptr);
  return host ? y.to_cpu() : y;
}

}  // namespace vision
}  // namespace rustorch

// ---------------------------------------------------------------- C shim
// C entry points for the ResNet-18 model (include/rustorch_b200_vision.h); a
// C++ exception becomes a status code with its message as the last error.
namespace rtb {
int set_error(int status, const std::string& msg);
}

extern "C" {

int rtb_resnet18_create(int device, uint64_t seed, int precision, void** handle) {
  if (!handle) return rtb::set_error(RTB_E_INVALID, "null handle out");
  try {
    *handle = new rustorch::vision::ResNet18(seed, device, precision);
    return RTB_OK;
  } catch (const std::exception& e) {
    *handle = nullptr;
    return rtb::set_error(RTB_E_CUDA, e.what());
  }
}

int rtb_resnet18_destroy(void* handle) {
  delete static_cast<rustorch::vision::ResNet18*>(handle);
  return RTB_OK;
}

int rtb_resnet18_forward(void* handle, int64_t batch, const float* x_nchw, float* logits,
                         void* stream) {
  if (!handle || batch <= 0 || !x_nchw || !logits) return RTB_E_INVALID;
  try {
    static_cast<rustorch::vision::ResNet18*>(handle)->forward_device(batch, x_nchw, logits, stream);
    return RTB_OK;
  } catch (const std::exception& e) {
    return rtb::set_error(RTB_E_CUDA, e.what());
  }
}

int64_t rtb_resnet18_num_params(void* handle) {
  return handle ? (int64_t) static_cast<rustorch::vision::ResNet18*>(handle)->num_params() : -1;
}

int rtb_resnet18_get_param(void* handle, int64_t index, float* host_out, int64_t* shape4) {
  if (!handle || index < 0) return RTB_E_INVALID;
  try {
    auto* net = static_cast<rustorch::vision::ResNet18*>(handle);
    if ((size_t)index >= net->num_params()) return RTB_E_INVALID;
    rustorch::Tensor t = net->param((size_t)index).to_cpu();
    for (int k = 0; k < 4; ++k) shape4[k] = k < (int)t.dim() ? (int64_t)t.shape()[k] : 1;
    if (host_out) {
      std::vector<float> v = t.data();
      std::memcpy(host_out, v.data(), v.size() * sizeof(float));
    }
    return RTB_OK;
  } catch (const std::exception& e) {
    return rtb::set_error(RTB_E_CUDA, e.what());
  }
}

int64_t rtb_resnet18_flops_per_image(void* handle) {
  return handle ? static_cast<rustorch::vision::ResNet18*>(handle)->flops_per_image() : -1;
}

}  // extern "C"
