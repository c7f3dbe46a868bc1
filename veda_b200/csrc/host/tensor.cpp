// veda::core on device memory. Follows src/libs/tensor/Tensor.cpp (views, reshape refusal,
// contiguous) with device storage from the stream-ordered pool.
#include "veda/tensor.hpp"

#include "veda_cuda.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <sstream>
#include <stdexcept>

namespace veda
{

namespace
{
thread_local veda_stream_t g_stream = nullptr;
}

veda_stream_t current_stream() { return g_stream; }
void set_current_stream(veda_stream_t stream) { g_stream = stream; }

void check(int status, const char* what)
{
    if (status == VEDA_OK)
    {
        return;
    }
    std::string msg = what ? std::string(what) + ": " : std::string();
    msg += veda_last_error();
    switch (status)
    {
    case VEDA_ERR_INVALID_ARGUMENT:
        throw std::invalid_argument(msg);
    case VEDA_ERR_OUT_OF_RANGE:
        throw std::out_of_range(msg);
    default:
        throw std::runtime_error(msg);
    }
}

namespace core
{

namespace
{
void cuda_check(cudaError_t err, const char* what)
{
    if (err != cudaSuccess)
    {
        throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(err));
    }
}

cudaStream_t cs() { return reinterpret_cast<cudaStream_t>(current_stream()); }

// The stream-ordered pool gives memory back to the system at every synchronisation unless told
// to keep it; a training step allocates the same working set every time, so keep all of it.
void configure_pool_once()
{
    static bool done[64] = {false};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64 || done[device])
    {
        return;
    }
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess)
    {
        uint64_t threshold = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    done[device] = true;
}
} // namespace

size_t dtype_size(DType d) { return d == DType::BF16 ? 2 : 4; }
const char* dtype_name(DType d) { return d == DType::BF16 ? "bf16" : "f32"; }

Shape::Shape(std::vector<size_t> dims) : dims_(std::move(dims))
{
    size_ = 1;
    for (size_t d : dims_)
    {
        size_ *= d;
    }
}

Shape::Shape(std::initializer_list<size_t> dims) : Shape(std::vector<size_t>(dims)) {}

size_t Shape::operator[](size_t i) const
{
    if (i >= dims_.size())
    {
        throw std::out_of_range("Shape: axis " + std::to_string(i) + " of rank " +
                                std::to_string(dims_.size()));
    }
    return dims_[i];
}

std::string Shape::to_string() const
{
    std::ostringstream os;
    os << "[";
    for (size_t i = 0; i < dims_.size(); ++i)
    {
        os << (i ? ", " : "") << dims_[i];
    }
    os << "]";
    return os.str();
}

std::vector<size_t> contiguous_strides(const Shape& shape)
{
    std::vector<size_t> s(shape.rank(), 1);
    for (size_t k = shape.rank(); k-- > 1;)
    {
        s[k - 1] = s[k] * shape[k];
    }
    return s;
}

Storage::Storage(size_t bytes, bool zero) : bytes_(bytes)
{
    if (bytes == 0)
    {
        return;
    }
    configure_pool_once();
    cuda_check(cudaMallocAsync(&data_, bytes, cs()), "Storage: cudaMallocAsync");
    if (zero)
    {
        cuda_check(cudaMemsetAsync(data_, 0, bytes, cs()), "Storage: cudaMemsetAsync");
    }
}

Storage::Storage(void* external, size_t bytes) : data_(external), bytes_(bytes), owned_(false) {}

void Storage::flush_mirror() const
{
    if (mirror_dirty_)
    {
        cuda_check(cudaDeviceSynchronize(), "Storage: host mirror write-back (synchronize)");
        cuda_check(cudaMemcpy(data_, mirror_.get(), bytes_, cudaMemcpyHostToDevice),
                   "Storage: host mirror write-back");
        mirror_dirty_ = false;
    }
    mirror_valid_ = false;   // the device may change the buffer from here on
}

void* Storage::data()
{
    if (mirror_)
    {
        flush_mirror();
    }
    return data_;
}

const void* Storage::data() const
{
    if (mirror_)
    {
        flush_mirror();
    }
    return data_;
}

unsigned char* Storage::host_mirror(bool writable) const
{
    if (!mirror_)
    {
        mirror_ = std::make_unique<unsigned char[]>(bytes_ > 0 ? bytes_ : 1);
    }
    if (!mirror_valid_ && !mirror_dirty_)
    {
        cuda_check(cudaDeviceSynchronize(), "Storage: host mirror (synchronize)");
        if (bytes_ > 0)
        {
            cuda_check(cudaMemcpy(mirror_.get(), data_, bytes_, cudaMemcpyDeviceToHost),
                       "Storage: host mirror");
        }
        mirror_valid_ = true;
    }
    if (writable)
    {
        mirror_dirty_ = true;
    }
    return mirror_.get();
}

Storage::~Storage()
{
    if (owned_ && data_ != nullptr && cudaFreeAsync(data_, cs()) != cudaSuccess)
    {
        // a destructor cannot throw: leave the error for the next check, and say which block
        std::fprintf(stderr, "veda: freeing %zu device bytes failed: %s\n", bytes_,
                     cudaGetErrorString(cudaPeekAtLastError()));
    }
}

Tensor::Tensor(Shape shape) : Tensor(std::move(shape), DType::F32) {}

Tensor::Tensor(Shape shape, DType dtype)
    : storage_(std::make_shared<Storage>(shape.size() * dtype_size(dtype), true)),
      shape_(std::move(shape)),
      strides_(contiguous_strides(shape_)),
      dtype_(dtype)
{
}

Tensor::Tensor(std::shared_ptr<Storage> storage, size_t offset, Shape shape,
               std::vector<size_t> strides, DType dtype)
    : storage_(std::move(storage)), offset_(offset), shape_(std::move(shape)),
      strides_(std::move(strides)), dtype_(dtype)
{
}

Tensor Tensor::empty(Shape shape, DType dtype)
{
    auto storage = std::make_shared<Storage>(shape.size() * dtype_size(dtype), false);
    std::vector<size_t> strides = contiguous_strides(shape);
    return Tensor(std::move(storage), 0, std::move(shape), std::move(strides), dtype);
}

Tensor Tensor::view(std::shared_ptr<Storage> storage, size_t offset, Shape shape, DType dtype)
{
    std::vector<size_t> strides = contiguous_strides(shape);
    return view(std::move(storage), offset, std::move(shape), std::move(strides), dtype);
}

Tensor Tensor::view(std::shared_ptr<Storage> storage, size_t offset, Shape shape,
                    std::vector<size_t> strides, DType dtype)
{
    if (!storage)
    {
        throw std::invalid_argument("Tensor::view: storage is null");
    }
    if (strides.size() != shape.rank())
    {
        throw std::invalid_argument("Tensor::view: shape " + shape.to_string() + " has rank " +
                                    std::to_string(shape.rank()) + " but " +
                                    std::to_string(strides.size()) + " strides");
    }
    size_t last = offset;
    for (size_t k = 0; k < shape.rank(); ++k)
    {
        if (shape[k] == 0)
        {
            last = offset;
            break;
        }
        last += (shape[k] - 1) * strides[k];
    }
    if (shape.size() > 0 && (last + 1) * dtype_size(dtype) > storage->bytes())
    {
        throw std::out_of_range("Tensor::view: shape " + shape.to_string() +
                                " runs past the end of its storage");
    }
    return Tensor(std::move(storage), offset, std::move(shape), std::move(strides), dtype);
}

Tensor Tensor::from_host(const std::vector<float>& values, Shape shape, DType dtype)
{
    if (values.size() != shape.size())
    {
        throw std::invalid_argument("Tensor::from_host: " + std::to_string(values.size()) +
                                    " values for shape " + shape.to_string());
    }
    Tensor f = Tensor::empty(shape, DType::F32);
    if (!values.empty())
    {
        cuda_check(cudaMemcpyAsync(f.data_ptr(), values.data(), values.size() * sizeof(float),
                                   cudaMemcpyHostToDevice, cs()),
                   "Tensor::from_host");
    }
    return dtype == DType::F32 ? f : to_dtype(f, dtype);
}

std::vector<float> Tensor::to_host() const
{
    const Tensor c = (is_contiguous() && dtype_ == DType::F32) ? *this : to_dtype(*this, DType::F32);
    std::vector<float> out(numel());
    if (!out.empty())
    {
        cuda_check(cudaMemcpyAsync(out.data(), c.data_ptr(), out.size() * sizeof(float),
                                   cudaMemcpyDeviceToHost, cs()),
                   "Tensor::to_host");
    }
    cuda_check(cudaStreamSynchronize(cs()), "Tensor::to_host: synchronize");
    return out;
}

float Tensor::at(std::initializer_list<size_t> indices) const
{
    if (indices.size() != rank())
    {
        throw std::out_of_range("Tensor::at: " + std::to_string(indices.size()) +
                                " indices for rank " + std::to_string(rank()));
    }
    size_t flat = offset_;
    size_t k = 0;
    for (size_t i : indices)
    {
        if (i >= shape_[k])
        {
            throw std::out_of_range("Tensor::at: index " + std::to_string(i) + " on axis " +
                                    std::to_string(k) + " of extent " +
                                    std::to_string(shape_[k]));
        }
        flat += i * strides_[k];
        ++k;
    }
    const Tensor one = view(storage_, flat, Shape({1}), dtype_);
    return one.to_host()[0];
}

bool Tensor::is_contiguous() const { return strides_ == contiguous_strides(shape_); }

Tensor Tensor::reshape(const Shape& new_shape) const
{
    if (new_shape.size() != numel())
    {
        throw std::invalid_argument("Tensor::reshape: " + shape_.to_string() + " has " +
                                    std::to_string(numel()) + " elements, " +
                                    new_shape.to_string() + " needs " +
                                    std::to_string(new_shape.size()));
    }
    if (!is_contiguous())
    {
        throw std::logic_error("Tensor::reshape: the tensor is not contiguous; call contiguous()");
    }
    return Tensor(storage_, offset_, new_shape, contiguous_strides(new_shape), dtype_);
}

Tensor Tensor::transpose(size_t a, size_t b) const
{
    if (a >= rank() || b >= rank())
    {
        throw std::out_of_range("Tensor::transpose: axis out of range");
    }
    std::vector<size_t> dims = shape_.dims();
    std::vector<size_t> strides = strides_;
    std::swap(dims[a], dims[b]);
    std::swap(strides[a], strides[b]);
    return Tensor(storage_, offset_, Shape(std::move(dims)), std::move(strides), dtype_);
}

Tensor Tensor::slice(size_t dim, size_t start, size_t count) const
{
    if (dim >= rank() || start + count > shape_[dim])
    {
        throw std::out_of_range("Tensor::slice: range outside the dimension");
    }
    std::vector<size_t> dims = shape_.dims();
    dims[dim] = count;
    return Tensor(storage_, offset_ + start * strides_[dim], Shape(std::move(dims)), strides_,
                  dtype_);
}

float* Tensor::data()
{
    if (dtype_ != DType::F32)
    {
        throw std::logic_error("Tensor::data: host element access is for fp32 tensors");
    }
    if (!storage_)
    {
        return nullptr;
    }
    return reinterpret_cast<float*>(storage_->host_mirror(true)) + offset_;
}

const float* Tensor::data() const
{
    if (dtype_ != DType::F32)
    {
        throw std::logic_error("Tensor::data: host element access is for fp32 tensors");
    }
    if (!storage_)
    {
        return nullptr;
    }
    return reinterpret_cast<const float*>(storage_->host_mirror(false)) + offset_;
}

void* Tensor::data_ptr() const
{
    if (!storage_)
    {
        return nullptr;
    }
    return static_cast<char*>(storage_->data()) + offset_ * dtype_size(dtype_);
}

int64_t Tensor::ld() const
{
    if (rank() < 2 || strides_.back() != 1)
    {
        throw std::invalid_argument("Tensor::ld: needs a rank >= 2 view with a contiguous last dim");
    }
    // rows of a [.., rows, cols] view flattened over the leading axes must be evenly strided
    for (size_t k = 0; k + 2 < rank(); ++k)
    {
        if (strides_[k] != strides_[k + 1] * shape_[k + 1])
        {
            throw std::invalid_argument("Tensor::ld: leading axes do not flatten");
        }
    }
    return static_cast<int64_t>(strides_[rank() - 2]);
}

Tensor to_dtype(const Tensor& tensor, DType dtype)
{
    Tensor out = Tensor::empty(tensor.shape(), dtype);
    if (tensor.numel() == 0)
    {
        return out;
    }
    std::vector<int64_t> shape(tensor.shape().dims().begin(), tensor.shape().dims().end());
    std::vector<int64_t> strides(tensor.strides().begin(), tensor.strides().end());
    if (shape.empty())
    {
        shape.push_back(1);
        strides.push_back(1);
    }
    check(veda_copy_strided(tensor.storage()->data(), static_cast<int>(tensor.dtype()),
                            strides.data(), static_cast<int64_t>(tensor.offset()), out.data_ptr(),
                            static_cast<int>(dtype), shape.data(), static_cast<int>(shape.size()),
                            current_stream()),
          "contiguous");
    return out;
}

Tensor contiguous(const Tensor& tensor) { return to_dtype(tensor, tensor.dtype()); }

} // namespace core
} // namespace veda
