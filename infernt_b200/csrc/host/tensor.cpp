// tensor.cpp — host/GPU buffer implementing include/tensor.h.
#include "tensor.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

namespace {
void cuda_or_throw(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}
}  // namespace

size_t dtype_size(DType dtype) {
    switch (dtype) {
        case DType::FP32: return 4;
        case DType::FP16: return 2;
        case DType::BF16: return 2;
        case DType::INT32: return 4;
        case DType::INT64: return 8;
        case DType::UINT8: return 1;
    }
    return 0;
}

const char* dtype_name(DType dtype) {
    switch (dtype) {
        case DType::FP32: return "FP32";
        case DType::FP16: return "FP16";
        case DType::BF16: return "BF16";
        case DType::INT32: return "INT32";
        case DType::INT64: return "INT64";
        case DType::UINT8: return "UINT8";
    }
    return "UNKNOWN";
}

const char* device_name(Device device) { return device == Device::CPU ? "CPU" : "CUDA"; }

Tensor::Tensor()
    : data_(nullptr), num_elements_(0), dtype_(DType::FP32), device_(Device::CPU), owns_data_(false) {}

Tensor::Tensor(const std::vector<int>& shape, DType dtype, Device device)
    : data_(nullptr), shape_(shape), num_elements_(1), dtype_(dtype), device_(device), owns_data_(true) {
    for (int s : shape_) {
        if (s <= 0) throw std::invalid_argument("Tensor dimensions must be positive");
        num_elements_ *= s;
    }
    compute_strides();
    allocate();
}

Tensor::~Tensor() { free_memory(); }

Tensor::Tensor(Tensor&& o) noexcept
    : data_(o.data_), shape_(std::move(o.shape_)), strides_(std::move(o.strides_)),
      num_elements_(o.num_elements_), dtype_(o.dtype_), device_(o.device_), owns_data_(o.owns_data_) {
    o.data_ = nullptr;
    o.num_elements_ = 0;
    o.owns_data_ = false;
}

Tensor& Tensor::operator=(Tensor&& o) noexcept {
    if (this != &o) {
        free_memory();
        data_ = o.data_;
        shape_ = std::move(o.shape_);
        strides_ = std::move(o.strides_);
        num_elements_ = o.num_elements_;
        dtype_ = o.dtype_;
        device_ = o.device_;
        owns_data_ = o.owns_data_;
        o.data_ = nullptr;
        o.num_elements_ = 0;
        o.owns_data_ = false;
    }
    return *this;
}

Tensor Tensor::zeros(const std::vector<int>& shape, DType dtype, Device device) {
    Tensor t(shape, dtype, device);
    if (device == Device::CPU)
        std::memset(t.data_, 0, t.size_bytes());
    else
        cuda_or_throw(cudaMemset(t.data_, 0, t.size_bytes()), "cudaMemset");
    return t;
}

Tensor Tensor::empty(const std::vector<int>& shape, DType dtype, Device device) {
    return Tensor(shape, dtype, device);
}

Tensor Tensor::to(Device target) const {
    if (target == device_) throw std::runtime_error("Tensor is already on the target device");
    Tensor r(shape_, dtype_, target);
    cuda_or_throw(cudaMemcpy(r.data_, data_, size_bytes(),
                             target == Device::CUDA ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToHost),
                  "cudaMemcpy");
    return r;
}

Tensor Tensor::clone() const {
    Tensor r(shape_, dtype_, device_);
    r.copy_from(*this);
    return r;
}

void Tensor::copy_from(const Tensor& src) {
    if (num_elements_ != src.num_elements_ || dtype_ != src.dtype_)
        throw std::runtime_error("Tensor shape/dtype mismatch in copy_from");
    if (device_ == Device::CPU && src.device_ == Device::CPU) {
        std::memcpy(data_, src.data_, size_bytes());
        return;
    }
    cudaMemcpyKind kind = cudaMemcpyDeviceToDevice;
    if (device_ == Device::CUDA && src.device_ == Device::CPU) kind = cudaMemcpyHostToDevice;
    if (device_ == Device::CPU && src.device_ == Device::CUDA) kind = cudaMemcpyDeviceToHost;
    cuda_or_throw(cudaMemcpy(data_, src.data_, size_bytes(), kind), "cudaMemcpy");
}

void* Tensor::data_ptr() { return data_; }
const void* Tensor::data_ptr() const { return data_; }

float* Tensor::data_as_float() {
    if (dtype_ != DType::FP32) throw std::runtime_error("Tensor is not FP32");
    return static_cast<float*>(data_);
}

const float* Tensor::data_as_float() const {
    if (dtype_ != DType::FP32) throw std::runtime_error("Tensor is not FP32");
    return static_cast<const float*>(data_);
}

int Tensor::dim() const { return static_cast<int>(shape_.size()); }
int Tensor::size(int d) const { return shape_.at(d); }
const std::vector<int>& Tensor::shape() const { return shape_; }
const std::vector<int>& Tensor::strides() const { return strides_; }
int64_t Tensor::num_elements() const { return num_elements_; }
size_t Tensor::size_bytes() const { return static_cast<size_t>(num_elements_) * dtype_size(dtype_); }
DType Tensor::dtype() const { return dtype_; }
Device Tensor::device() const { return device_; }
bool Tensor::is_cuda() const { return device_ == Device::CUDA; }
bool Tensor::is_cpu() const { return device_ == Device::CPU; }
bool Tensor::is_valid() const { return data_ != nullptr && num_elements_ > 0; }

Tensor Tensor::reshape(const std::vector<int>& new_shape) const {
    int64_t n = 1;
    for (int s : new_shape) n *= s;
    if (n != num_elements_) throw std::runtime_error("Reshape: element count mismatch");
    Tensor r;
    r.data_ = data_;
    r.shape_ = new_shape;
    r.num_elements_ = num_elements_;
    r.dtype_ = dtype_;
    r.device_ = device_;
    r.owns_data_ = false;
    r.compute_strides();
    return r;
}

void Tensor::print_info(const std::string& label) const {
    if (!label.empty()) std::printf("%s: ", label.c_str());
    std::printf("Tensor(shape=[");
    for (int i = 0; i < dim(); ++i) std::printf(i ? ", %d" : "%d", shape_[i]);
    std::printf("], dtype=%s, device=%s, elements=%lld, bytes=%zu)\n", dtype_name(dtype_),
                device_name(device_), (long long)num_elements_, size_bytes());
}

void Tensor::print_data(int max_elements) const {
    if (!is_cpu()) {
        std::printf("[Tensor on GPU - copy to CPU to print data]\n");
        return;
    }
    if (dtype_ != DType::FP32) {
        std::printf("[print_data supports FP32 only]\n");
        return;
    }
    const float* d = static_cast<const float*>(data_);
    const int n = num_elements_ < max_elements ? (int)num_elements_ : max_elements;
    std::printf("[");
    for (int i = 0; i < n; ++i) std::printf(i ? ", %.6f" : "%.6f", d[i]);
    if (n < num_elements_) std::printf(", ... (%lld more)", (long long)(num_elements_ - n));
    std::printf("]\n");
}

void Tensor::allocate() {
    const size_t bytes = size_bytes();
    if (bytes == 0) return;
    if (device_ == Device::CPU) {
        data_ = std::malloc(bytes);
        if (!data_) throw std::runtime_error("CPU memory allocation failed");
    } else {
        cudaError_t e = cudaMalloc(&data_, bytes);
        if (e != cudaSuccess) {
            data_ = nullptr;
            throw std::runtime_error(std::string("GPU memory allocation failed: ") + cudaGetErrorString(e));
        }
    }
}

void Tensor::free_memory() {
    if (data_ && owns_data_) {
        if (device_ == Device::CPU)
            std::free(data_);
        else
            cudaFree(data_);
    }
    data_ = nullptr;
}

void Tensor::compute_strides() {
    strides_.assign(shape_.size(), 1);
    for (int i = (int)shape_.size() - 2; i >= 0; --i) strides_[i] = strides_[i + 1] * shape_[i + 1];
}
