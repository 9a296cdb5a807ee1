// tensor.cpp — the Tensor of include/tensor.h: a move-only buffer on the
// host or the current GPU.
//
// Storage: host buffers are 64-byte aligned (vector loads in host code),
// device buffers come from cudaMalloc.  Every transfer goes through one
// routine that picks the route from the two devices: host to host is a
// memcpy; a transfer with a device end is issued on the legacy default
// stream (the stream the reference's launch_* kernels use), so it is
// ordered after every kernel launched there, and the call waits for it only
// when a host buffer is read or written (device-to-device copies return at
// once, like a kernel launch).  Views (reshape) share the storage without
// owning it.
#include "tensor.h"

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <string>

namespace {

[[noreturn]] void fail(const std::string& what) { throw std::runtime_error("Tensor: " + what); }

void check_cuda(cudaError_t e, const char* call) {
    if (e != cudaSuccess) fail(std::string(call) + " failed (" + cudaGetErrorString(e) + ")");
}

constexpr size_t kHostAlign = 64;

void* storage_alloc(Device dev, size_t bytes) {
    if (bytes == 0) return nullptr;
    if (dev == Device::CPU) {
        const size_t rounded = (bytes + kHostAlign - 1) / kHostAlign * kHostAlign;
        void* p = std::aligned_alloc(kHostAlign, rounded);
        if (!p) fail("host allocation of " + std::to_string(bytes) + " bytes failed");
        return p;
    }
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail("device allocation of " + std::to_string(bytes) + " bytes failed (" + cudaGetErrorString(e) + ")");
    }
    return p;
}

void storage_release(Device dev, void* p) {
    if (!p) return;
    if (dev == Device::CPU)
        std::free(p);
    else
        cudaFree(p);
}

// bytes from src (on src_dev) to dst (on dst_dev)
void transfer(void* dst, Device dst_dev, const void* src, Device src_dev, size_t bytes) {
    if (bytes == 0) return;
    if (dst_dev == Device::CPU && src_dev == Device::CPU) {
        std::memcpy(dst, src, bytes);
        return;
    }
    const cudaMemcpyKind kind = dst_dev == Device::CUDA
                                    ? (src_dev == Device::CUDA ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice)
                                    : cudaMemcpyDeviceToHost;
    check_cuda(cudaMemcpyAsync(dst, src, bytes, kind, cudaStreamLegacy), "cudaMemcpyAsync");
    if (kind != cudaMemcpyDeviceToDevice) check_cuda(cudaStreamSynchronize(cudaStreamLegacy), "cudaStreamSynchronize");
}

int64_t element_count(const std::vector<int>& shape) {
    int64_t n = 1;
    for (size_t i = 0; i < shape.size(); ++i) {
        if (shape[i] <= 0) fail("extent " + std::to_string(shape[i]) + " of dimension " + std::to_string(i) +
                                " is not positive");
        if (n > std::numeric_limits<int64_t>::max() / shape[i]) fail("element count overflows");
        n *= shape[i];
    }
    return n;
}

}  // namespace

size_t dtype_size(DType dtype) {
    switch (dtype) {
        case DType::UINT8: return 1;
        case DType::FP16:
        case DType::BF16: return 2;
        case DType::FP32:
        case DType::INT32: return 4;
        case DType::INT64: return 8;
    }
    return 0;
}

const char* dtype_name(DType dtype) {
    static const char* const names[] = {"FP32", "FP16", "BF16", "INT32", "INT64", "UINT8"};
    const int i = static_cast<int>(dtype);
    return i >= 0 && i < 6 ? names[i] : "?";
}

const char* device_name(Device device) { return device == Device::CUDA ? "CUDA" : "CPU"; }

Tensor::Tensor()
    : data_(nullptr), num_elements_(0), dtype_(DType::FP32), device_(Device::CPU), owns_data_(false) {}

Tensor::Tensor(const std::vector<int>& shape, DType dtype, Device device)
    : data_(nullptr), shape_(shape), num_elements_(element_count(shape)), dtype_(dtype), device_(device),
      owns_data_(true) {
    compute_strides();
    allocate();
}

Tensor::~Tensor() { free_memory(); }

Tensor::Tensor(Tensor&& other) noexcept
    : data_(nullptr), num_elements_(0), dtype_(DType::FP32), device_(Device::CPU), owns_data_(false) {
    *this = std::move(other);
}

Tensor& Tensor::operator=(Tensor&& other) noexcept {
    if (this == &other) return *this;
    free_memory();
    data_ = other.data_;
    shape_.swap(other.shape_);
    strides_.swap(other.strides_);
    num_elements_ = other.num_elements_;
    dtype_ = other.dtype_;
    device_ = other.device_;
    owns_data_ = other.owns_data_;
    // the source keeps nothing: it is an empty, invalid tensor
    other.data_ = nullptr;
    other.shape_.clear();
    other.strides_.clear();
    other.num_elements_ = 0;
    other.owns_data_ = false;
    return *this;
}

Tensor Tensor::empty(const std::vector<int>& shape, DType dtype, Device device) { return Tensor(shape, dtype, device); }

Tensor Tensor::zeros(const std::vector<int>& shape, DType dtype, Device device) {
    Tensor t(shape, dtype, device);
    if (device == Device::CUDA) {
        // complete before return: the caller may hand the buffer to kernels
        // on any stream
        check_cuda(cudaMemsetAsync(t.data_, 0, t.size_bytes(), cudaStreamLegacy), "cudaMemsetAsync");
        check_cuda(cudaStreamSynchronize(cudaStreamLegacy), "cudaStreamSynchronize");
    } else
        std::memset(t.data_, 0, t.size_bytes());
    return t;
}

Tensor Tensor::to(Device target_device) const {
    if (target_device == device_)
        fail(std::string("to(): the tensor already lives on ") + device_name(device_));
    Tensor out(shape_, dtype_, target_device);
    transfer(out.data_, target_device, data_, device_, size_bytes());
    return out;
}

Tensor Tensor::clone() const {
    Tensor out(shape_, dtype_, device_);
    transfer(out.data_, device_, data_, device_, size_bytes());
    return out;
}

void Tensor::copy_from(const Tensor& src) {
    if (src.dtype_ != dtype_)
        fail(std::string("copy_from(): dtype ") + dtype_name(src.dtype_) + " into " + dtype_name(dtype_));
    if (src.num_elements_ != num_elements_)
        fail("copy_from(): " + std::to_string(src.num_elements_) + " elements into " + std::to_string(num_elements_));
    transfer(data_, device_, src.data_, src.device_, size_bytes());
}

void* Tensor::data_ptr() { return data_; }
const void* Tensor::data_ptr() const { return data_; }

float* Tensor::data_as_float() {
    if (dtype_ != DType::FP32) fail(std::string("data_as_float(): the tensor holds ") + dtype_name(dtype_));
    return static_cast<float*>(data_);
}

const float* Tensor::data_as_float() const { return const_cast<Tensor*>(this)->data_as_float(); }

uint16_t* Tensor::data_as_bf16() {
    if (dtype_ != DType::BF16) fail(std::string("data_as_bf16(): the tensor holds ") + dtype_name(dtype_));
    return static_cast<uint16_t*>(data_);
}

const uint16_t* Tensor::data_as_bf16() const { return const_cast<Tensor*>(this)->data_as_bf16(); }

int Tensor::dim() const { return static_cast<int>(shape_.size()); }
int Tensor::size(int d) const {
    if (d < 0 || d >= dim()) fail("size(" + std::to_string(d) + ") of a " + std::to_string(dim()) + "-d tensor");
    return shape_[d];
}
const std::vector<int>& Tensor::shape() const { return shape_; }
const std::vector<int>& Tensor::strides() const { return strides_; }
int64_t Tensor::num_elements() const { return num_elements_; }
size_t Tensor::size_bytes() const { return static_cast<size_t>(num_elements_) * dtype_size(dtype_); }
DType Tensor::dtype() const { return dtype_; }
Device Tensor::device() const { return device_; }
bool Tensor::is_cuda() const { return device_ == Device::CUDA; }
bool Tensor::is_cpu() const { return device_ == Device::CPU; }
bool Tensor::is_valid() const { return data_ && num_elements_ > 0; }

Tensor Tensor::reshape(const std::vector<int>& new_shape) const {
    if (element_count(new_shape) != num_elements_)
        fail("reshape(): " + std::to_string(element_count(new_shape)) + " elements from " +
             std::to_string(num_elements_));
    Tensor view;
    view.data_ = data_;
    view.shape_ = new_shape;
    view.num_elements_ = num_elements_;
    view.dtype_ = dtype_;
    view.device_ = device_;
    view.owns_data_ = false;
    view.compute_strides();
    return view;
}

void Tensor::print_info(const std::string& label) const {
    std::string dims;
    for (int i = 0; i < dim(); ++i) dims += (i ? "x" : "") + std::to_string(shape_[i]);
    std::printf("%s%s%s %s on %s, %lld elements (%zu bytes)\n", label.c_str(), label.empty() ? "" : ": ",
                dims.empty() ? "[]" : dims.c_str(), dtype_name(dtype_), device_name(device_),
                static_cast<long long>(num_elements_), size_bytes());
}

void Tensor::print_data(int max_elements) const {
    if (device_ != Device::CPU || dtype_ != DType::FP32 || !data_) {
        std::printf("(print_data shows FP32 host tensors; this one is %s on %s)\n", dtype_name(dtype_),
                    device_name(device_));
        return;
    }
    const float* v = static_cast<const float*>(data_);
    const int64_t n = num_elements_ < max_elements ? num_elements_ : (max_elements < 0 ? 0 : max_elements);
    std::string line = "{";
    char buf[32];
    for (int64_t i = 0; i < n; ++i) {
        std::snprintf(buf, sizeof(buf), "%s%g", i ? " " : "", v[i]);
        line += buf;
    }
    if (n < num_elements_) line += " +" + std::to_string(num_elements_ - n) + " more";
    std::printf("%s}\n", line.c_str());
}

void Tensor::allocate() { data_ = storage_alloc(device_, size_bytes()); }

void Tensor::free_memory() {
    if (owns_data_) storage_release(device_, data_);
    data_ = nullptr;
    owns_data_ = false;
}

void Tensor::compute_strides() {
    strides_.resize(shape_.size());
    int stride = 1;
    for (size_t i = shape_.size(); i-- > 0;) {
        strides_[i] = stride;
        stride *= shape_[i];
    }
}
