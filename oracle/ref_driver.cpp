// ref_driver.cpp - a C entry layer over the reference's own CPU kernels, for pinning the oracle and for the CPU baseline.
//
// TEST INFRASTRUCTURE ONLY. oracle/Makefile compiles this file together with the reference sources where they lie
// (src/kernels.cpp, src/weights.cpp, and src/decoders.cpp, which this translation unit includes so that its file-local
// helpers norm_rows, rms_heads, gelu_tanh and silu can be called) into oracle/_ref/libidolref.so. Nothing of the
// reference is copied; the library only exists where the reference tree is present.
#include "decoders.cpp"  // NOLINT: the reference's translation unit, for its file-local helpers

#include <omp.h>

#include <cstdint>
#include <cstring>
#include <exception>
#include <string>

extern "C" int orc_q8_to_panels(const std::uint8_t* q8, int out, int in, std::uint8_t* blob);
extern "C" std::int64_t orc_panel_blob_bytes(int out, int in);

namespace {
thread_local std::string g_error;
}

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

void ref_set_threads(int n) { omp_set_num_threads(n); }
int ref_max_threads() { return omp_get_max_threads(); }

// Wraps Q8_0 blocks (out rows of in/32 blocks) as the reference's PackedLinear through the GGUF->native conversion
// (tools/gguf_to_decoder.py:16-40) and quantized_linear (src/kernels.cpp:516-533). Returns nullptr on error.
void* ref_q8_linear_create(const std::uint8_t* q8, const float* bias, int out, int in) {
    try {
        std::vector<std::uint8_t> blob((std::size_t)orc_panel_blob_bytes(out, in));
        if (orc_q8_to_panels(q8, out, in, blob.data()) != 0) {
            g_error = "Q8_0 scale cannot be represented exactly in the native layout";
            return nullptr;
        }
        std::vector<float> b(bias ? std::vector<float>(bias, bias + out) : std::vector<float>((std::size_t)out, 0.0f));
        return new idol::detail::PackedLinear(idol::detail::quantized_linear(std::move(blob), b, out, in, 8, 32));
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

// Wraps a raw panel blob with any supported bits/group (the reference test's reference_quantize output).
void* ref_blob_linear_create(const std::uint8_t* blob, std::int64_t nbytes, const float* bias, int out, int in,
                             int bits, int group) {
    try {
        std::vector<std::uint8_t> b(blob, blob + nbytes);
        std::vector<float> bb(bias, bias + out);
        return new idol::detail::PackedLinear(idol::detail::quantized_linear(std::move(b), bb, out, in, bits, group));
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

void ref_linear_free(void* h) { delete static_cast<idol::detail::PackedLinear*>(h); }

// mode 0 forces the float kernel (production: tools/idol_generate.py:356), 1 the AVX-VNNI integer kernel.
void ref_gemm(void* h, const float* a, int m, int n_offset, int n, const float* residual, int gelu, float* c,
              int mode) {
    idol::detail::set_quant_kernel(mode);
    idol::detail::gemm_packed(a, m, *static_cast<idol::detail::PackedLinear*>(h), n_offset, n, residual, gelu != 0, c);
}

void ref_dequantize(void* h, float* w) {
    const auto v = idol::detail::dequantize_linear(*static_cast<idol::detail::PackedLinear*>(h));
    std::memcpy(w, v.data(), v.size() * sizeof(float));
}

void ref_norm_rows(const float* x, float* y, int rows, int dim, float eps, const float* gamma, const float* beta,
                   const float* shift, const float* scale) {
    idol::norm_rows(x, y, rows, dim, eps, gamma, beta, shift, scale);
}

void ref_layer_norm(const float* x, int rows, int dim, const float* gamma, const float* beta, float* y) {
    idol::detail::layer_norm(x, rows, dim, gamma, beta, y);
}

void ref_rms_heads(float* x, int rows, int ld, int heads, int hd, const float* gamma) {
    idol::rms_heads(x, rows, ld, heads, hd, gamma);
}

void ref_gelu_tanh(float* x, std::int64_t count) { idol::gelu_tanh(x, (std::size_t)count); }

float ref_silu(float x) { return idol::silu(x); }

float ref_gelu_scalar(float x) { return idol::detail::gelu_scalar(x); }

void ref_attention(const float* q, int lq, int ldq, const float* k, const float* v, int lk, int ldkv, int heads,
                   int head_dim, float* out, int dim) {
    idol::detail::attention(q, lq, ldq, k, v, lk, ldkv, heads, head_dim, out, dim);
}

// The reference's decoders, loaded from a native export directory (manifest.txt + weights.bin, src/weights.cpp:25-104),
// through their public API (include/idol/decoders.hpp). Returns nullptr on error (ref_last_error says why).
void* ref_decoders_open(const char* dir) {
    try {
        return new idol::Decoders(dir);
    } catch (const std::exception& e) {
        g_error = e.what();
        return nullptr;
    }
}

void ref_decoders_free(void* h) { delete static_cast<idol::Decoders*>(h); }

// mode selects the quantized GEMM kernel as in ref_gemm: 0 the float kernel that production forces
// (tools/idol_generate.py:356), 1 the AVX-VNNI integer kernel (the library's default on such CPUs).
void ref_gaussian_features(void* h, const float* points, int rows, const float* cond, int cond_rows, float* out,
                           int mode) {
    idol::detail::set_quant_kernel(mode);
    static_cast<idol::Decoders*>(h)->gaussian_features(points, rows, cond, cond_rows, out);
}

void ref_octree_logits(void* h, const float* x, int rows, float resolution, const float* cond, int cond_rows,
                       float* out, int mode) {
    idol::detail::set_quant_kernel(mode);
    static_cast<idol::Decoders*>(h)->octree_logits(x, rows, resolution, cond, cond_rows, out);
}

// Decoders::sample_anchors into points [num_points, 3]; returns num_points, or -1 (ref_last_error says why).
int ref_sample_anchors(void* h, const float* cond, int cond_rows, int num_points, int level, std::uint64_t seed,
                       float* points, int mode) {
    try {
        idol::detail::set_quant_kernel(mode);
        const std::vector<float> p =
            static_cast<idol::Decoders*>(h)->sample_anchors(cond, cond_rows, num_points, level, seed);
        std::memcpy(points, p.data(), p.size() * sizeof(float));
        return (int)(p.size() / 3);
    } catch (const std::exception& e) {
        g_error = e.what();
        return -1;
    }
}

// Decoders::to_gaussians, copied out of the GaussianCloud: xyz, f_dc, scale [rows * per_anchor, 3], rotation [.., 4],
// opacity [..].
void ref_to_gaussians(void* h, const float* anchors, int rows, const float* features, float* xyz, float* f_dc,
                      float* scale, float* rotation, float* opacity) {
    const idol::GaussianCloud c = static_cast<idol::Decoders*>(h)->to_gaussians(anchors, rows, features);
    std::memcpy(xyz, c.xyz.data(), c.xyz.size() * sizeof(float));
    std::memcpy(f_dc, c.f_dc.data(), c.f_dc.size() * sizeof(float));
    std::memcpy(scale, c.scale.data(), c.scale.size() * sizeof(float));
    std::memcpy(rotation, c.rotation.data(), c.rotation.size() * sizeof(float));
    std::memcpy(opacity, c.opacity.data(), c.opacity.size() * sizeof(float));
}

}  // extern "C"
