// modarith.hpp -- host modular arithmetic for NTT plans: 64-bit modular
// products, Miller-Rabin, the reference's root convention and Shoup
// quotients.  Shared by the RNS ABI and the main-ABI NTT.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>

namespace cubf::modarith {

using u64 = std::uint64_t;
using u128 = unsigned __int128;

inline u64 mulmod(u64 a, u64 b, u64 q) { return static_cast<u64>(static_cast<u128>(a) * b % q); }

inline u64 powmod(u64 b, u64 e, u64 q) {
    u64 r = 1 % q;
    b %= q;
    for (; e; e >>= 1, b = mulmod(b, b, q))
        if (e & 1) r = mulmod(r, b, q);
    return r;
}

// Deterministic Miller-Rabin for 64-bit integers: trial division by the
// primes to 37, then the seven-witness set that is exact below 2^64
// (the reference's is_prime, src/reference.cpp:522-562).
inline bool is_prime(u64 n) {
    if (n < 2) return false;
    for (u64 p : {2ull, 3ull, 5ull, 7ull, 11ull, 13ull, 17ull, 19ull, 23ull, 29ull, 31ull, 37ull})
        if (n % p == 0) return n == p;
    u64 d = n - 1;
    int s = 0;
    while (!(d & 1)) {
        d >>= 1;
        ++s;
    }
    for (u64 a : {2ull, 325ull, 9375ull, 28178ull, 450775ull, 9780504ull, 1795265022ull}) {
        if (a % n == 0) continue;
        u64 x = powmod(a, d, n);
        if (x == 1 || x == n - 1) continue;
        bool ok = false;
        for (int r = 1; r < s; ++r) {
            x = mulmod(x, x, n);
            if (x == n - 1) {
                ok = true;
                break;
            }
        }
        if (!ok) return false;
    }
    return true;
}

// The primitive 2^log_n-th root of unity the reference's plans and oracle use
// (find_primitive_power_of_two_root, src/reference.cpp:564-582): the first
// candidate c = 2, 3, ... whose power c^((q-1)/2^log_n) has order exactly
// 2^log_n.  Throws std::invalid_argument when q is not a prime with
// 2^log_n | q - 1.
inline u64 primitive_root_of_two_power(unsigned log_n, u64 q) {
    if (log_n == 0 || log_n >= 63) throw std::invalid_argument("log_n must be in [1, 62]");
    if (!is_prime(q)) throw std::invalid_argument("modulus must be prime");
    const u64 n = u64{1} << log_n;
    if ((q - 1) % n != 0) throw std::invalid_argument("modulus - 1 is not divisible by the requested NTT length");
    for (u64 c = 2; c < (u64{1} << 20); ++c) {
        const u64 r = powmod(c, (q - 1) / n, q);
        if (powmod(r, n, q) == 1 && powmod(r, n >> 1, q) != 1) return r;
    }
    throw std::runtime_error("could not find a primitive power-of-two root");
}

// Shoup quotient floor(w 2^64 / q) of a constant w < q.
// The primitive root of an arbitrary order the reference's Bluestein NTT
// uses (src/bluestein_ntt.cu:42-57): the first candidate c = 2, 3, ... below
// 2^20 whose power c^((q - 1) / order) has exactly that order (checked
// against every prime factor of the order).
inline u64 primitive_root_of_order(u64 order, u64 q) {
    if (!is_prime(q)) throw std::invalid_argument("Bluestein NTT modulus must be prime");
    if (order < 2 || (q - 1) % order != 0)
        throw std::invalid_argument("modulus does not admit the required 2N-th Bluestein root");
    u64 factors[64];
    int nf = 0;
    u64 v = order;
    for (u64 f = 2; f <= v / f; ++f) {
        if (v % f) continue;
        factors[nf++] = f;
        while (v % f == 0) v /= f;
    }
    if (v > 1) factors[nf++] = v;
    for (u64 c = 2; c < (u64{1} << 20); ++c) {
        const u64 r = powmod(c, (q - 1) / order, q);
        bool primitive = powmod(r, order, q) == 1;
        for (int i = 0; i < nf && primitive; ++i) primitive = powmod(r, order / factors[i], q) != 1;
        if (primitive) return r;
    }
    throw std::runtime_error("could not find the required Bluestein NTT root");
}

inline u64 shoup(u64 w, u64 q) { return static_cast<u64>((static_cast<u128>(w) << 64) / q); }

inline std::size_t bitrev(std::size_t x, int bits) {
    std::size_t r = 0;
    for (int i = 0; i < bits; ++i, x >>= 1) r = (r << 1) | (x & 1);
    return r;
}

// Cyclic root schedule of the tile kernels: entry k = 2^s + i (stage s,
// butterfly block i) holds base^(bitrev_s(i) * 2^(L-1-s)); entry 0 is 1.
// With base = omega the Cooley-Tukey passes compute the DFT over omega into
// bit-reversed order; the Gentleman-Sande passes with the same table compute
// it from bit-reversed input.  roots and quots hold 2^log_n entries.
inline void cyclic_root_table(int log_n, u64 q, u64 base, u64* roots, u64* quots) {
    const std::size_t n = std::size_t{1} << log_n;
    // powers base^e for e < n/2 suffice: bitrev_s(i) * 2^(L-1-s) < 2^(L-1)
    u64* pw = quots;  // scratch: quots is overwritten below
    pw[0] = 1;
    for (std::size_t e = 1; e < n / 2; ++e) pw[e] = mulmod(pw[e - 1], base, q);
    roots[0] = 1;
    for (int s = 0; s < log_n; ++s)
        for (std::size_t i = 0; i < (std::size_t{1} << s); ++i)
            roots[(std::size_t{1} << s) + i] = pw[bitrev(i, s) << (log_n - 1 - s)];
    for (std::size_t k = 0; k < n; ++k) quots[k] = shoup(roots[k], q);
}

}  // namespace cubf::modarith
