// Compile-only stand-in for the XLA FFI header, used solely to build the reference's kernel
// sources (cuda/*.cu of sokrypton/colabfold-legacy-kernels) as a legacy comparator under
// oracle/_ref -- TEST INFRASTRUCTURE, never part of the product.
//
// It declares just what the reference's handler bodies use: an error value with the three
// factories, a typed buffer that wraps a device pointer and its dimensions, a result wrapper,
// and a handler-definition macro that drops the binding (the comparator calls the handler
// bodies directly, e.g. VoltaMmaImpl, with buffers built from raw pointers).  Nothing here is
// taken from XLA; the real header is not available in this environment.
#pragma once

#include <cstdint>
#include <initializer_list>
#include <string>
#include <utility>

namespace xla {
namespace ffi {

enum class DataType { F16, F32, U8 };

template <DataType T>
struct NativeType;
template <>
struct NativeType<DataType::F16> {
    using type = uint16_t;
};
template <>
struct NativeType<DataType::F32> {
    using type = float;
};
template <>
struct NativeType<DataType::U8> {
    using type = uint8_t;
};

class Error {
  public:
    Error() = default;
    static Error Success() { return Error(); }
    static Error InvalidArgument(std::string m) { return Error(1, std::move(m)); }
    static Error Internal(std::string m) { return Error(2, std::move(m)); }
    int code() const { return code_; }
    const std::string& message() const { return msg_; }

  private:
    Error(int c, std::string m) : code_(c), msg_(std::move(m)) {}
    int code_ = 0;
    std::string msg_;
};

struct Dims {
    int64_t d[4] = {0, 0, 0, 0};
    int n = 0;
    size_t size() const { return static_cast<size_t>(n); }
    int64_t operator[](size_t i) const { return d[i]; }
};

template <DataType T>
class Buffer {
  public:
    using Native = typename NativeType<T>::type;
    Buffer(const void* data, std::initializer_list<int64_t> dims)
        : data_(const_cast<void*>(data)) {
        for (int64_t v : dims) {
            dims_.d[dims_.n++] = v;
        }
    }
    Dims dimensions() const { return dims_; }
    Native* typed_data() const { return static_cast<Native*>(data_); }

  private:
    void* data_;
    Dims dims_;
};

template <typename B>
class Result {
  public:
    explicit Result(B* b) : b_(b) {}
    B* operator->() const { return b_; }

  private:
    B* b_;
};

} // namespace ffi
} // namespace xla

// The comparator calls the handler bodies directly; the symbol and its binding are not needed.
#define XLA_FFI_DEFINE_HANDLER_SYMBOL(...)
