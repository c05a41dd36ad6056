// binding_test.cpp — TEST INFRASTRUCTURE. Compiles the servoflow-side binding
// (integration/sfb_servoflow.hpp) against servoflow's own headers and exposes
// it to the GPU tests as plain C functions: each wraps device pointers in
// sf::Tensor views (the way servoflow's backend hands tensors to
// CUDABackend::attention / dequantize) and calls the binding. Built by
// `make -C oracle binding` into oracle/_ref/libsfb_binding_test.so.
#include <cstring>
#include <exception>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "sfb_servoflow.hpp"

namespace {

thread_local std::string g_msg;

sf::Tensor view(const void* p, const std::vector<int64_t>& shape, int dtype) {
    auto st = std::make_shared<sf::Storage>(const_cast<void*>(p), 0, sf::kCUDA0, nullptr);
    sf::Shape s;
    switch (shape.size()) {
        case 1: s = sf::Shape({shape[0]}); break;
        case 2: s = sf::Shape({shape[0], shape[1]}); break;
        case 3: s = sf::Shape({shape[0], shape[1], shape[2]}); break;
        default: s = sf::Shape({shape[0], shape[1], shape[2], shape[3]}); break;
    }
    return sf::Tensor(st, s, static_cast<sf::DType>(dtype));
}

// 0 = ok, 1 = std::invalid_argument, 2 = std::runtime_error, 3 = other.
template <typename F> int guarded(F&& f) {
    try {
        f();
        g_msg.clear();
        return 0;
    } catch (const std::invalid_argument& e) {
        g_msg = e.what();
        return 1;
    } catch (const std::runtime_error& e) {
        g_msg = e.what();
        return 2;
    } catch (...) {
        g_msg = "unknown exception";
        return 3;
    }
}

}  // namespace

extern "C" {

const char* sfbind_last_message(void) { return g_msg.c_str(); }

// Contiguous BHSD q/k/v/out; v_dtype may differ from dtype (fp16 V cache).
// mask (optional): mask_ndim dims in mask_shape, contiguous, dtype mask_dtype.
int sfbind_attention(const void* q, const void* k, const void* v, void* out, int dtype, int v_dtype,
                     int B, int H, int Lq, int Lk, int D, const void* mask, int mask_dtype, int mask_ndim,
                     const int64_t* mask_shape, float scale, int causal, void* stream) {
    return guarded([&] {
        sf::Tensor Q = view(q, {B, H, Lq, D}, dtype), K = view(k, {B, H, Lk, D}, dtype);
        sf::Tensor V = view(v, {B, H, Lk, D}, v_dtype), O = view(out, {B, H, Lq, D}, dtype);
        std::unique_ptr<sf::Tensor> M;
        if (mask != nullptr)
            M.reset(new sf::Tensor(view(mask, std::vector<int64_t>(mask_shape, mask_shape + mask_ndim), mask_dtype)));
        sfb_servoflow::attention(Q, K, V, O, M.get(), scale, causal != 0, static_cast<cudaStream_t>(stream));
    });
}

int sfbind_dequantize(const void* in, const void* scale, int scale_dtype, long scale_numel, void* out,
                      int out_dtype, long rows, long cols, void* stream) {
    return guarded([&] {
        sf::Tensor I = view(in, {rows, cols}, static_cast<int>(sf::DType::Int8));
        sf::Tensor S = view(scale, {scale_numel}, scale_dtype);
        sf::Tensor O = view(out, {rows, cols}, out_dtype);
        sfb_servoflow::dequantize(I, S, O, static_cast<cudaStream_t>(stream));
    });
}

}  // extern "C"
