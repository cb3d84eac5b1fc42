// sb_dequant_f16: packed 2/4/8-bit weights -> f16, bit-exact with the
// reference's dq_f16 (gemma4_150/kernels_dsl.py:2101-2138): one thread per
// packed 32-bit word, value i of the word at bit BITS*i, w = f16(s * (q - ZP))
// with the product formed in f32 and rounded once to nearest-even.
#include "common.cuh"

namespace {

template <int BITS, bool SCALE_F16>
__global__ void __launch_bounds__(256) dequant_kernel(const uint32_t* __restrict__ packed,
                                                      const void* __restrict__ scales,
                                                      __half* __restrict__ out, int n_in, int group,
                                                      int64_t n_words) {
  constexpr int VPW = 32 / BITS;  // values per word
  constexpr uint32_t MASK = (1u << BITS) - 1u;
  constexpr float ZP = static_cast<float>(1 << (BITS - 1));
  const int words_per_row = n_in / VPW;
  const int groups_per_row = n_in / group;
  for (int64_t wi = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; wi < n_words;
       wi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = wi / words_per_row;
    const int col0 = static_cast<int>(wi - row * words_per_row) * VPW;
    const int64_t si = row * groups_per_row + col0 / group;  // a word never straddles a group
    const float s = SCALE_F16 ? __half2float(static_cast<const __half*>(scales)[si])
                              : static_cast<const float*>(scales)[si];
    const uint32_t w = __ldg(packed + wi);
    __half2 v[VPW / 2];
#pragma unroll
    for (int i = 0; i < VPW; i += 2) {
      const float q0 = static_cast<float>((w >> (BITS * i)) & MASK) - ZP;
      const float q1 = static_cast<float>((w >> (BITS * (i + 1))) & MASK) - ZP;
      v[i / 2] = __halves2half2(__float2half_rn(__fmul_rn(s, q0)), __float2half_rn(__fmul_rn(s, q1)));
    }
    __half2* dst = reinterpret_cast<__half2*>(out + row * n_in + col0);
#pragma unroll
    for (int i = 0; i < VPW / 2; ++i) dst[i] = v[i];
  }
}

template <int BITS>
int launch(const void* packed, const void* scales, bool f16_scale, void* out, int n_out, int n_in,
           int group, cudaStream_t s) {
  const int64_t n_words = static_cast<int64_t>(n_out) * (n_in / (32 / BITS));
  if (n_words == 0) return SB_OK;
  const int64_t want = (n_words + 255) / 256;
  const int grid = static_cast<int>(want < 65535 * 8 ? want : 65535 * 8);
  if (f16_scale)
    dequant_kernel<BITS, true><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(packed), scales,
                                                    static_cast<__half*>(out), n_in, group, n_words);
  else
    dequant_kernel<BITS, false><<<grid, 256, 0, s>>>(static_cast<const uint32_t*>(packed), scales,
                                                     static_cast<__half*>(out), n_in, group, n_words);
  return sb::launch_status("dequant_kernel");
}

}  // namespace

extern "C" int sb_dequant_f16(const void* packed, int bits, const void* scales, int scale_dtype, int group,
                              void* out, int n_out, int n_in, void* stream) {
  SB_CHECK_ARG(bits == 2 || bits == 4 || bits == 8, "sb_dequant_f16: bits must be 2, 4 or 8 (got %d)", bits);
  SB_CHECK_ARG(n_out >= 0 && n_in >= 0, "sb_dequant_f16: negative shape");
  SB_CHECK_ARG(scale_dtype == SB_SCALE_F16 || scale_dtype == SB_SCALE_F32, "sb_dequant_f16: bad scale dtype");
  SB_CHECK_ARG(n_in % (32 / bits) == 0, "sb_dequant_f16: n_in=%d must be a multiple of %d", n_in, 32 / bits);
  SB_CHECK_ARG(group > 0 && n_in % group == 0 && (group % 32 == 0 || group == n_in),
               "sb_dequant_f16: group=%d must divide n_in=%d and be a multiple of 32 (or n_in)", group, n_in);
  if (n_out == 0 || n_in == 0) return SB_OK;
  SB_CHECK_ARG(packed && scales && out, "sb_dequant_f16: null pointer");
  if (!sb::aligned(packed, 4) || !sb::aligned(out, 4))
    return sb::fail(SB_ERR_ALIGN, "sb_dequant_f16: packed and out must be 4-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool f16s = scale_dtype == SB_SCALE_F16;
  switch (bits) {
    case 2: return launch<2>(packed, scales, f16s, out, n_out, n_in, group, s);
    case 4: return launch<4>(packed, scales, f16s, out, n_out, n_in, group, s);
    default: return launch<8>(packed, scales, f16s, out, n_out, n_in, group, s);
  }
}
