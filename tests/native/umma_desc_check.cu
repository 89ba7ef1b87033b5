// Host-only check (test infrastructure): the tcgen05 descriptors geode_b200/csrc/umma.cuh builds by hand against CuTe's
// own builders (make_umma_desc / make_instr_desc) for the same operand layouts. Prints one line per case and exits 1
// on any difference. Built and run by tests/test_umma_desc.py.
#include <cstdio>

#include <cute/tensor.hpp>
#include <cute/arch/mma_sm100_desc.hpp>
#include <cute/atom/mma_traits_sm100.hpp>

#include "../../geode_b200/csrc/umma.cuh"

using namespace cute;

template <int Rows, int Lbo, int Sbo>
int check_smem() {
    // int8, K-major, no swizzle: ((8, Rows/8), (16, 2)) : ((16, Sbo), (1, Lbo)) in elements (bytes)
    auto layout = make_layout(make_shape(make_shape(Int<8>{}, Int<Rows / 8>{}), make_shape(Int<16>{}, Int<2>{})),
                              make_stride(make_stride(Int<16>{}, Int<Sbo>{}), make_stride(Int<1>{}, Int<Lbo>{})));
    auto t = make_tensor(make_smem_ptr(reinterpret_cast<uint8_t *>(0)), layout);
    const uint64_t want = static_cast<uint64_t>(UMMA::make_umma_desc<UMMA::Major::K>(t));
    const uint64_t got = gcu::umma_smem_desc(0, Lbo, Sbo);
    std::printf("smem rows %d lbo %d sbo %d: cute %016llx ours %016llx\n", Rows, Lbo, Sbo, (unsigned long long)want,
                (unsigned long long)got);
    return want != got;
}

// int8, K-major, 128-byte swizzle (CuTe's Layout_K_SW128_Atom tiled to Rows x 128): an atom of 8 rows x 128 bytes (four
// K = 32 steps), row groups 1024 bytes apart
template <int Rows>
int check_smem_sw128() {
    auto layout = tile_to_shape(UMMA::Layout_K_SW128_Atom<uint8_t>{}, make_shape(Int<Rows>{}, Int<128>{}));
    auto t = make_tensor(make_smem_ptr(reinterpret_cast<uint8_t *>(0)), layout);
    const uint64_t want = static_cast<uint64_t>(UMMA::make_umma_desc<UMMA::Major::K>(t));
    const uint64_t got = gcu::umma_smem_desc_sw128(0, 1024);
    std::printf("smem sw128 rows %d: cute %016llx ours %016llx\n", Rows, (unsigned long long)want, (unsigned long long)got);
    return want != got;
}

template <int M, int N, class A, class B>
int check_idesc() {
    const uint32_t want = static_cast<uint32_t>(
        UMMA::make_instr_desc<A, B, int32_t, M, N, UMMA::Major::K, UMMA::Major::K>());
    const uint32_t got = gcu::umma_idesc_i8(M, N, std::is_same<A, int8_t>::value, std::is_same<B, int8_t>::value);
    std::printf("idesc M %d N %d: cute %08x ours %08x\n", M, N, want, got);
    return want != got;
}

int main() {
    int bad = 0;
    bad += check_smem<128, 128, 256>();
    bad += check_smem<8, 128, 0>();   // (one group of 8 rows: the stride between groups is unused, CuTe writes 0)
    bad += check_smem<64, 128, 256>();
    bad += check_smem<128, 2048, 16>();
    bad += check_smem_sw128<128>();
    bad += check_smem_sw128<64>();
    bad += check_idesc<128, 8, uint8_t, int8_t>();
    bad += check_idesc<128, 16, uint8_t, int8_t>();
    bad += check_idesc<128, 64, uint8_t, int8_t>();
    bad += check_idesc<128, 256, uint8_t, int8_t>();
    bad += check_idesc<64, 8, int8_t, int8_t>();
    std::printf(bad ? "MISMATCH\n" : "ok\n");
    return bad ? 1 : 0;
}
