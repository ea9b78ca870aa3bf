// quantize.cu -- per-output-channel symmetric INT8 quantizer on the GPU.
//
// Same arithmetic as quantize_per_channel (bench_int8.py:19-24 and
// int8_decoder.py:45-56 in the reference):
//   absmax = |W[m,:]|.amax() in bf16 (exact: abs and max do not round)
//   scale  = fp32(bf16(absmax / 127))  (torch divides a bf16 tensor by a python
//            scalar in fp32 and rounds the quotient to bf16; fp32 division and
//            multiplication by fp32(1/127) give the same bf16 for every finite
//            bf16 input, which
//            tests/test_oracle_golden.py::test_scale_division_unambiguous_for_all_bf16
//            checks exhaustively)
//   scale  = max(scale, 1e-12)
//   q      = clamp(rint(fp32(W) / scale), -128, 127)  (IEEE division, round half even)
// This file is compiled without --use_fast_math and uses __fdiv_rn explicitly.
#include "common.cuh"

namespace mq {

__global__ void __launch_bounds__(256) quantize_rows_kernel(const __nv_bfloat16* __restrict__ w,
                                                            int64_t M, int64_t K,
                                                            int8_t* __restrict__ q,
                                                            float* __restrict__ scale) {
    const int64_t row = blockIdx.x;
    if (row >= M) return;
    const __nv_bfloat16* wr = w + row * K;
    float amax = 0.f;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x)
        amax = fmaxf(amax, fabsf(__bfloat162float(wr[k])));
    amax = warp_max(amax);
    __shared__ float red[8];
    __shared__ float s_scale;
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) m = fmaxf(m, red[i]);
        float s = __bfloat162float(__float2bfloat16_rn(__fdiv_rn(m, 127.0f)));
        s = fmaxf(s, 1e-12f);
        s_scale = s;
        scale[row] = s;
    }
    __syncthreads();
    const float s = s_scale;
    int8_t* qr = q + row * K;
    for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
        float v = rintf(__fdiv_rn(__bfloat162float(wr[k]), s));
        v = fminf(fmaxf(v, -128.f), 127.f);
        qr[k] = (int8_t)(int)v;
    }
}

}  // namespace mq

extern "C" int mq_quantize_per_channel(const void* w_bf16, int64_t M, int64_t K, int8_t* q_out,
                                       float* scale_out, cudaStream_t stream) {
    if (!w_bf16 || !q_out || !scale_out || M <= 0 || K <= 0) return MQ_ERR_ARG;
    if (M > 0x7fffffffLL) return MQ_ERR_SIZE;
    mq::quantize_rows_kernel<<<(unsigned)M, 256, 0, stream>>>((const __nv_bfloat16*)w_bf16, M, K, q_out,
                                                            scale_out);
    return (int)cudaGetLastError();
}
