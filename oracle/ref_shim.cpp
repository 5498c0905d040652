// ref_shim.cpp -- extern "C" entry points over the reference's own CPU oracles.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the unmodified reference sources src/butterfly_reference.cpp and
// src/reference.cpp (read in place from the reference tree) into
// oracle/_ref/libcubf_ref.so.  The shim only marshals arrays in and out of the
// std::vector signatures declared in include/cuntt/butterfly.hpp:377-390 and
// include/cuntt/ntt.hpp:427-430; all arithmetic is the reference's.
// It is used to pin oracle/cubf_oracle.c and, in bench.py, as the timed CPU
// baseline ("kind": "reference"), spreading independent transforms over
// std::threads.
#include <cuntt/butterfly.hpp>
#include <cuntt/ntt.hpp>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {
template <class F>
void parallel_for(std::size_t count, int threads, F&& body) {
    if (threads <= 1 || count <= 1) {
        for (std::size_t i = 0; i < count; ++i) body(i);
        return;
    }
    std::atomic<std::size_t> next{0};
    std::vector<std::thread> pool;
    const int used = static_cast<int>(std::min<std::size_t>(count, static_cast<std::size_t>(threads)));
    for (int t = 0; t < used; ++t)
        pool.emplace_back([&] {
            for (std::size_t i; (i = next.fetch_add(1)) < count;) body(i);
        });
    for (auto& th : pool) th.join();
}

std::uint16_t round_bf16(double value) {
    const __nv_bfloat16 b = __double2bfloat16(value);
    std::uint16_t bits;
    std::memcpy(&bits, &b, 2);
    return bits;
}
double widen_bf16(std::uint16_t bits) {
    std::uint32_t u = static_cast<std::uint32_t>(bits) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}
}  // namespace

extern "C" {

int cubf_ref_fft_c32(float* data, std::size_t n, std::size_t batch, int inverse, int normalize, int threads) {
    try {
        parallel_for(batch, threads, [&](std::size_t b) {
            std::vector<cuntt::Complex32> v(n);
            std::memcpy(v.data(), data + 2 * n * b, n * sizeof(cuntt::Complex32));
            cuntt::reference_fft(v, inverse != 0, normalize != 0);
            std::memcpy(data + 2 * n * b, v.data(), n * sizeof(cuntt::Complex32));
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

int cubf_ref_fft_c64(double* data, std::size_t n, std::size_t batch, int inverse, int normalize, int threads) {
    try {
        parallel_for(batch, threads, [&](std::size_t b) {
            std::vector<cuntt::Complex64> v(n);
            for (std::size_t i = 0; i < n; ++i) v[i] = {data[2 * (n * b + i)], data[2 * (n * b + i) + 1]};
            cuntt::reference_fft(v, inverse != 0, normalize != 0);
            for (std::size_t i = 0; i < n; ++i) {
                data[2 * (n * b + i)] = v[i].real;
                data[2 * (n * b + i) + 1] = v[i].imag;
            }
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

// widen bf16 -> reference_fwht<double> -> x scale -> round to bf16 (RNE).
int cubf_ref_fwht_bf16_final(const std::uint16_t* in, std::uint16_t* out, std::size_t n, std::size_t batch,
                             int inverse, int normalize, double scale, int threads) {
    try {
        parallel_for(batch, threads, [&](std::size_t b) {
            std::vector<double> v(n);
            for (std::size_t i = 0; i < n; ++i) v[i] = widen_bf16(in[n * b + i]);
            cuntt::reference_fwht(v, inverse != 0, normalize != 0);
            for (std::size_t i = 0; i < n; ++i) out[n * b + i] = round_bf16(v[i] * scale);
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

int cubf_ref_fwht_f32(float* data, std::size_t n, std::size_t batch, int inverse, int normalize, int threads) {
    try {
        parallel_for(batch, threads, [&](std::size_t b) {
            std::vector<float> v(data + n * b, data + n * (b + 1));
            cuntt::reference_fwht(v, inverse != 0, normalize != 0);
            std::copy(v.begin(), v.end(), data + n * b);
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

int cubf_ref_zeta_u32(std::uint32_t* data, std::size_t n, std::size_t batch, int superset, int inverse, int threads) {
    try {
        parallel_for(batch, threads, [&](std::size_t b) {
            std::vector<std::uint32_t> v(data + n * b, data + n * (b + 1));
            if (superset)
                cuntt::reference_superset_zeta(v, inverse != 0);
            else
                cuntt::reference_subset_zeta(v, inverse != 0);
            std::copy(v.begin(), v.end(), data + n * b);
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

int cubf_ref_is_prime(std::uint64_t value) { return cuntt::is_prime(value) ? 1 : 0; }

std::uint64_t cubf_ref_find_root(unsigned log_n, std::uint64_t q) {
    try {
        return cuntt::find_primitive_power_of_two_root(log_n, q);
    } catch (...) {
        return 0;
    }
}

// Forward negacyclic NTT, natural input, bit-reversed output, built from the
// reference's cyclic reference_ntt: twist by psi^j (psi = primitive 2n-th root
// found by find_primitive_power_of_two_root(log n + 1, q), whose square is the
// root reference_ntt uses), cyclic NTT, then bit-reverse the output.
int cubf_ref_negacyclic_ntt(const std::uint64_t* in, std::uint64_t* out, unsigned log_n, std::size_t count,
                            const std::uint64_t* moduli, int threads) {
    try {
        const std::size_t n = std::size_t{1} << log_n;
        parallel_for(count, threads, [&](std::size_t p) {
            const std::uint64_t q = moduli[p];
            const std::uint64_t psi = cuntt::find_primitive_power_of_two_root(log_n + 1, q);
            std::vector<std::uint64_t> v(in + n * p, in + n * (p + 1));
            std::uint64_t twist = 1;
            for (auto& x : v) {
                x = static_cast<std::uint64_t>((static_cast<unsigned __int128>(x) * twist) % q);
                twist = static_cast<std::uint64_t>((static_cast<unsigned __int128>(twist) * psi) % q);
            }
            cuntt::reference_ntt(v, q, false);
            for (std::size_t j = 0; j < n; ++j) {
                std::size_t r = 0, x = j;
                for (unsigned b = 0; b < log_n; ++b, x >>= 1) r = (r << 1) | (x & 1);
                out[n * p + r] = v[j];
            }
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

// The reference's cyclic reference_ntt (src/reference.cpp:584-630) on each of
// `batch` packed transforms: natural in, natural out, root
// find_primitive_power_of_two_root(log n, q), inverse scaled by n^-1.
int cubf_ref_ntt_cyclic(std::uint64_t* data, std::size_t n, std::size_t batch, std::uint64_t q, int inverse,
                        int threads) {
    try {
        parallel_for(batch, threads, [&](std::size_t b) {
            std::vector<std::uint64_t> v(data + n * b, data + n * (b + 1));
            cuntt::reference_ntt(v, q, inverse != 0);
            std::copy(v.begin(), v.end(), data + n * b);
        });
    } catch (...) {
        return 1;
    }
    return 0;
}

// The reference's structured 2x2 butterfly (reference_structured_2x2,
// src/butterfly_reference.cpp:541-591); mats: 4 doubles per matrix.
int cubf_ref_structured_f32(float* data, std::size_t n, std::size_t batch, const double* mats, std::size_t count,
                            int inverse) {
    try {
        std::vector<cuntt::ButterflyMatrix2x2> ms(count);
        for (std::size_t i = 0; i < count; ++i) ms[i] = {mats[4 * i], mats[4 * i + 1], mats[4 * i + 2], mats[4 * i + 3]};
        for (std::size_t b = 0; b < batch; ++b) {
            std::vector<float> v(data + n * b, data + n * (b + 1));
            cuntt::reference_structured_2x2(v, ms, inverse != 0);
            std::copy(v.begin(), v.end(), data + n * b);
        }
    } catch (...) {
        return 1;
    }
    return 0;
}

int cubf_ref_abi_version(void) { return 3; }
}
