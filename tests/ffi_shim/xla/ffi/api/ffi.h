// Test-only stand-in for the XLA FFI header, used by tests/test_ffi_handlers.py to compile
// colabfold-legacy-kernels_b200/csrc/ffi_handlers.cc where jax (and its header) is absent.
//
// It provides the handful of types the handlers use, with plain semantics (a buffer is a data
// pointer, a dtype and dimensions), and a handler-definition macro that checks at compile time
// that each binding (Ctx / Arg / Ret / Attr, in order) has exactly the parameter list of its
// handler function.  Nothing here is XLA code; it stands in for it only in this test.
#pragma once

#include <cstdint>
#include <initializer_list>
#include <string>
#include <type_traits>
#include <utility>

namespace xla {
namespace ffi {

enum class DataType { F16, BF16, F32, U8 };

template <DataType T>
struct NativeType;
template <>
struct NativeType<DataType::F16> {
    using type = uint16_t;
};
template <>
struct NativeType<DataType::BF16> {
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

inline Dims make_dims(std::initializer_list<int64_t> dims) {
    Dims r;
    for (int64_t v : dims) {
        r.d[r.n++] = v;
    }
    return r;
}

class AnyBuffer {
  public:
    AnyBuffer(void* data, DataType t, std::initializer_list<int64_t> dims)
        : data_(data), type_(t), dims_(make_dims(dims)) {}
    DataType element_type() const { return type_; }
    Dims dimensions() const { return dims_; }
    void* untyped_data() const { return data_; }

  private:
    void* data_;
    DataType type_;
    Dims dims_;
};

template <DataType T>
class Buffer {
  public:
    Buffer(void* data, std::initializer_list<int64_t> dims) : data_(data), dims_(make_dims(dims)) {}
    Dims dimensions() const { return dims_; }
    typename NativeType<T>::type* typed_data() const {
        return static_cast<typename NativeType<T>::type*>(data_);
    }

  private:
    void* data_;
    Dims dims_;
};

template <typename T>
class Result {
  public:
    explicit Result(T v) : v_(std::move(v)) {}
    T& operator*() { return v_; }
    T* operator->() { return &v_; }

  private:
    T v_;
};

template <typename T>
struct PlatformStream {};
struct DeviceOrdinal {};
struct Traits {
    static constexpr int kCmdBufferCompatible = 1;
};

template <typename C>
struct CtxParam;
template <typename T>
struct CtxParam<PlatformStream<T>> {
    using type = T;
};
template <>
struct CtxParam<DeviceOrdinal> {
    using type = int32_t;
};

// The parameter list a binding describes, in order.
template <typename... Ps>
struct Binding {
    template <typename C>
    Binding<Ps..., typename CtxParam<C>::type> Ctx() const {
        return {};
    }
    template <typename A>
    Binding<Ps..., A> Arg() const {
        return {};
    }
    template <typename R>
    Binding<Ps..., Result<R>> Ret() const {
        return {};
    }
    template <typename T>
    Binding<Ps..., T> Attr(const char*) const {
        return {};
    }
    using Fn = Error (*)(Ps...);
};

struct Ffi {
    static Binding<> Bind() { return {}; }
};

} // namespace ffi
} // namespace xla

#define XLA_FFI_DEFINE_HANDLER_SYMBOL(fn, impl, binding, ...)                                      \
    static_assert(std::is_same<decltype(&impl), typename decltype(binding)::Fn>::value,          \
                  #fn ": the binding does not match the parameters of " #impl);                    \
    extern "C" __attribute__((visibility("default"))) int fn##_bound() { return 1; }
