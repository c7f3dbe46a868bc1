// veda::core — the reference's Tensor API (src/libs/tensor/Tensor.h:26-97, Shape.h, Storage.h)
// with storage in GPU memory and a dtype.
//
// As in the reference a Tensor is storage + offset + shape + strides: views (reshape, transpose,
// slice) share storage and cost nothing; contiguous() materialises. What changes:
//   * Storage is device memory from a stream-ordered pool (cudaMallocAsync on the current veda
//     stream), so allocation per op, which the reference's tape does, stays cheap;
//   * every Tensor has a DType: F32 (the reference's only arithmetic type) or BF16;
//   * element access from the host (at(), to_host(), data()) copies through PCIe and synchronises
//     — meant for tests, exactly like the reference's at() and data() are meant for them. data()
//     returns a pointer into a host mirror of the storage, filled from the device when it is
//     asked for and written back before the next device access after a writable data() call.
// Errors keep the reference's exception types: std::invalid_argument for bad shapes and
// arguments, std::out_of_range for bad indices and views, std::logic_error for reshaping a
// non-contiguous view, std::runtime_error for device failures.
#pragma once

#include <cstddef>
#include <cstdint>
#include <initializer_list>
#include <memory>
#include <ostream>
#include <string>
#include <vector>

typedef struct CUstream_st* veda_stream_t;

namespace veda
{

// The stream every veda op launches on (per thread; default: the legacy default stream).
veda_stream_t current_stream();
void set_current_stream(veda_stream_t stream);

// Throws the exception type the reference uses for the status code of a C-ABI call.
void check(int status, const char* what = nullptr);

namespace core
{

enum class DType
{
    F32 = 0,
    BF16 = 1
};

size_t dtype_size(DType d);
const char* dtype_name(DType d);

class Shape
{
public:
    Shape() = default;
    explicit Shape(std::vector<size_t> dims);
    Shape(std::initializer_list<size_t> dims);

    size_t rank() const noexcept { return dims_.size(); }
    size_t size() const noexcept { return size_; }
    size_t operator[](size_t i) const;
    const std::vector<size_t>& dims() const noexcept { return dims_; }
    bool operator==(const Shape& other) const noexcept { return dims_ == other.dims_; }
    bool operator!=(const Shape& other) const noexcept { return !(*this == other); }
    std::string to_string() const;

private:
    std::vector<size_t> dims_;
    size_t size_ = 1;
};

inline std::ostream& operator<<(std::ostream& os, const Shape& shape)
{
    return os << shape.to_string();
}

std::vector<size_t> contiguous_strides(const Shape& shape);

// A device buffer. Freed (stream-ordered) when the last Tensor viewing it goes away.
class Storage
{
public:
    explicit Storage(size_t bytes, bool zero = true);
    // Wraps memory owned elsewhere (not freed).
    Storage(void* external, size_t bytes);
    ~Storage();
    Storage(const Storage&) = delete;
    Storage& operator=(const Storage&) = delete;

    // Device address. If the host mirror may have been written since the last device access,
    // it is copied back first (synchronously).
    void* data();
    const void* data() const;
    size_t bytes() const noexcept { return bytes_; }
    // Host mirror of the whole buffer for Tensor::data(): filled from the device (after a device
    // synchronisation) unless it already holds the current contents; `writable` means the caller
    // may change it, so the next device access copies it back.
    unsigned char* host_mirror(bool writable) const;

private:
    void flush_mirror() const;
    void* data_ = nullptr;
    size_t bytes_ = 0;
    bool owned_ = true;
    mutable std::unique_ptr<unsigned char[]> mirror_;
    mutable bool mirror_valid_ = false;
    mutable bool mirror_dirty_ = false;
};

class Tensor
{
public:
    Tensor() = default;
    // Zero-filled fp32 storage, like the reference's Tensor(Shape).
    explicit Tensor(Shape shape);
    Tensor(Shape shape, DType dtype);
    // Uninitialised storage, for outputs an op overwrites completely.
    static Tensor empty(Shape shape, DType dtype = DType::F32);
    static Tensor view(std::shared_ptr<Storage> storage, size_t offset, Shape shape, DType dtype);
    static Tensor view(std::shared_ptr<Storage> storage, size_t offset, Shape shape,
                       std::vector<size_t> strides, DType dtype);
    // Host <-> device.
    static Tensor from_host(const std::vector<float>& values, Shape shape,
                            DType dtype = DType::F32);
    std::vector<float> to_host() const;

    const Shape& shape() const noexcept { return shape_; }
    const std::vector<size_t>& strides() const noexcept { return strides_; }
    size_t rank() const noexcept { return shape_.rank(); }
    size_t numel() const noexcept { return shape_.size(); }
    size_t offset() const noexcept { return offset_; }
    DType dtype() const noexcept { return dtype_; }
    bool defined() const noexcept { return storage_ != nullptr; }
    const std::shared_ptr<Storage>& storage() const noexcept { return storage_; }

    // Reads one element (a device-to-host copy; synchronises).
    float at(std::initializer_list<size_t> indices) const;
    // The reference's host element access (Tensor.h:76-77) for fp32 tensors: a host pointer to
    // this view's first element, strides as in strides(). It points into the storage's host
    // mirror (see Storage::host_mirror); device work queued before the call is waited for, and
    // writes through the non-const form reach the device before its next use there.
    float* data();
    const float* data() const;
    bool is_contiguous() const;
    Tensor reshape(const Shape& new_shape) const;
    Tensor transpose(size_t a, size_t b) const;
    Tensor slice(size_t dim, size_t start, size_t count) const;

    // Device address of the first element.
    void* data_ptr() const;
    // Row stride in elements of a 2-D view whose last dim is contiguous.
    int64_t ld() const;

private:
    Tensor(std::shared_ptr<Storage> storage, size_t offset, Shape shape,
           std::vector<size_t> strides, DType dtype);

    std::shared_ptr<Storage> storage_;
    size_t offset_ = 0;
    Shape shape_;
    std::vector<size_t> strides_;
    DType dtype_ = DType::F32;
};

// A dense copy of any view, in the requested dtype (default: the source's).
Tensor contiguous(const Tensor& tensor);
Tensor to_dtype(const Tensor& tensor, DType dtype);

} // namespace core
} // namespace veda
