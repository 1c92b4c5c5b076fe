// ref_w4a8_harness.cpp — extern "C" access to the reference test's own symmetric W4A8
// ("sdot5") checker, compiled in place from the reference tree (oracle/Makefile) into
// oracle/_ref/libtqref.so.
//
// TEST INFRASTRUCTURE ONLY.  The sdot5 kernels are aarch64-only, so on x86 the
// reference pins their arithmetic only through its test-side restatement
// matvec_i4_w4a8_naive (tests/test_matvec_i4.cpp:252-306), the symmetric packer
// pack_i4_rtn_symmetric (:403-438) and the inputs of random_vec (:144-152).  Those
// helpers live in an anonymous namespace of that test file, so this file includes the
// test translation unit itself (its TEST cases register with the header-only test
// framework and are never run) and exports the three helpers unchanged.
#include "test_matvec_i4.cpp"

extern "C" {

// y = matvec_i4_w4a8_naive(packed, x) for an [out_dim x in_dim] matrix in the i4 layout.
void tqref_matvec_i4_w4a8_naive(const uint8_t *w, const float *x, float *y, int out_dim,
                                int in_dim, int group_size) {
    const int groups = (in_dim + group_size - 1) / group_size;
    const size_t bytes = (size_t)out_dim * groups * (4 + group_size / 2);
    const std::vector<uint8_t> packed(w, w + bytes);
    const std::vector<float> xv(x, x + in_dim);
    const std::vector<float> out = matvec_i4_w4a8_naive(packed, xv, out_dim, in_dim, group_size);
    std::memcpy(y, out.data(), sizeof(float) * (size_t)out_dim);
}

// pack_i4_rtn_symmetric(w): zero = 8, scale = max|w| / 7 per group; dst holds
// out_dim * ceil(in_dim / G) * (4 + G/2) bytes.
void tqref_pack_i4_rtn_symmetric(const float *w, int out_dim, int in_dim, int group_size,
                                 uint8_t *dst) {
    const std::vector<float> wv(w, w + (size_t)out_dim * in_dim);
    const std::vector<uint8_t> p = pack_i4_rtn_symmetric(wv, out_dim, in_dim, group_size);
    std::memcpy(dst, p.data(), p.size());
}

// random_vec(n, seed): the test's N(0,1) inputs (std::mt19937 + normal_distribution).
void tqref_random_vec(size_t n, uint32_t seed, float *out) {
    const std::vector<float> v = random_vec(n, seed);
    std::memcpy(out, v.data(), sizeof(float) * n);
}

}  // extern "C"
