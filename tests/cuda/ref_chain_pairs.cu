// Test-only CUDA source: runs the scalar and the packed (f16x2/bf16x2) forms of
// the reference rounding chain on the same inputs so a test can compare their
// bits.  Compiled by tests/test_gpu_ref_chain.py with nvcc; not part of the library.
#include <cstdint>
#include "../../cann_operator_challenge_august_b200/csrc/common.cuh"

using namespace cgdr;

// in: [n][5] = u0, u1, a0, a1, gate  -> out: [n][4] = vn bits scalar, vd bits scalar, vn packed, vd packed
__global__ void epi1_pairs(const float* in, uint32_t* out, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = in + 5 * i;
    const float vn0 = ref_vnew(x[0], x[2]), vn1 = ref_vnew(x[1], x[3]);
    const float vd0 = ref_vdecay(vn0, x[4]), vd1 = ref_vdecay(vn1, x[4]);
    __half2 vnh = __floats2half2_rn(vn0, vn1);
    __nv_bfloat162 vdb = __floats2bfloat162_rn(vd0, vd1);
    uint32_t pn, pd;
    ref_vnew_vdecay_x2(x[0], x[1], x[2], x[3], __float2half2_rn(x[4]), pn, pd);
    out[4 * i + 0] = *reinterpret_cast<uint32_t*>(&vnh);
    out[4 * i + 1] = *reinterpret_cast<uint32_t*>(&vdb);
    out[4 * i + 2] = pn;
    out[4 * i + 3] = pd;
}

// in: [n][5] = s0, s1, a0, a1, alpha -> out: [n][4] = s0', s1' scalar, s0', s1' packed (fp32 bits)
__global__ void epi2_pairs(const float* in, uint32_t* out, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = in + 5 * i;
    float p0 = x[0], p1 = x[1];
    ref_state_x2(p0, p1, x[2], x[3], __float2half2_rn(x[4]));
    out[4 * i + 0] = __float_as_uint(ref_state(x[0], x[4], x[2]));
    out[4 * i + 1] = __float_as_uint(ref_state(x[1], x[4], x[3]));
    out[4 * i + 2] = __float_as_uint(p0);
    out[4 * i + 3] = __float_as_uint(p1);
}

// The chains without saturations, on inputs inside their stated domains:
// in: [n][5] = u0, u1, a0, a1, gate -> out: [n][4] = vn, vd bits scalar, vn, vd bits fast
__global__ void epi1_pairs_fast(const float* in, uint32_t* out, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = in + 5 * i;
    const float vn0 = ref_vnew(x[0], x[2]), vn1 = ref_vnew(x[1], x[3]);
    const float vd0 = ref_vdecay(vn0, x[4]), vd1 = ref_vdecay(vn1, x[4]);
    __half2 vnh = __floats2half2_rn(vn0, vn1);
    __nv_bfloat162 vdb = __floats2bfloat162_rn(vd0, vd1);
    uint32_t pn, pd;
    ref_vnew_vdecay_x2_fast(x[0], x[1], x[2], x[3], __float2half2_rn(x[4]), pn, pd);
    out[4 * i + 0] = *reinterpret_cast<uint32_t*>(&vnh);
    out[4 * i + 1] = *reinterpret_cast<uint32_t*>(&vdb);
    out[4 * i + 2] = pn;
    out[4 * i + 3] = pd;
}

// in: [n][5] = s0, s1, a0, a1, alpha -> out: [n][4] = s0', s1' scalar, s0', s1' fast (fp32 bits)
__global__ void epi2_pairs_fast(const float* in, uint32_t* out, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = in + 5 * i;
    float p0 = x[0], p1 = x[1];
    ref_state_x2_fast(p0, p1, h2_bits(ref_gemm_to_f16x2(x[2], x[3])), __float2half2_rn(x[4]));
    out[4 * i + 0] = __float_as_uint(ref_state(x[0], x[4], x[2]));
    out[4 * i + 1] = __float_as_uint(ref_state(x[1], x[4], x[3]));
    out[4 * i + 2] = __float_as_uint(p0);
    out[4 * i + 3] = __float_as_uint(p1);
}

// in: [n][5] = s0, s1 (bf16 values), a0, a1, alpha -> out: scalar s0', s1', then the fp32 values
// of the bf16 pair ref_state_bits_fast returns
__global__ void epi2_pairs_bits(const float* in, uint32_t* out, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = in + 5 * i;
    const __nv_bfloat162 sb = __floats2bfloat162_rn(x[0], x[1]);
    const uint32_t r = ref_state_bits_fast(*reinterpret_cast<const uint32_t*>(&sb),
                                           h2_bits(ref_gemm_to_f16x2(x[2], x[3])), __float2half2_rn(x[4]));
    out[4 * i + 0] = __float_as_uint(ref_state(x[0], x[4], x[2]));
    out[4 * i + 1] = __float_as_uint(ref_state(x[1], x[4], x[3]));
    out[4 * i + 2] = r << 16;
    out[4 * i + 3] = r & 0xffff0000u;
}

extern "C" int run_pairs(int which, const float* host_in, uint32_t* host_out, int n)
{
    float* din = nullptr;
    uint32_t* dout = nullptr;
    if (cudaMalloc(&din, sizeof(float) * 5 * n) != cudaSuccess) return 1;
    if (cudaMalloc(&dout, sizeof(uint32_t) * 4 * n) != cudaSuccess) return 2;
    cudaMemcpy(din, host_in, sizeof(float) * 5 * n, cudaMemcpyHostToDevice);
    if (which == 1)
        epi1_pairs<<<(n + 255) / 256, 256>>>(din, dout, n);
    else if (which == 2)
        epi2_pairs<<<(n + 255) / 256, 256>>>(din, dout, n);
    else if (which == 3)
        epi1_pairs_fast<<<(n + 255) / 256, 256>>>(din, dout, n);
    else if (which == 4)
        epi2_pairs_fast<<<(n + 255) / 256, 256>>>(din, dout, n);
    else
        epi2_pairs_bits<<<(n + 255) / 256, 256>>>(din, dout, n);
    cudaError_t e = cudaDeviceSynchronize();
    cudaMemcpy(host_out, dout, sizeof(uint32_t) * 4 * n, cudaMemcpyDeviceToHost);
    cudaFree(din);
    cudaFree(dout);
    return e == cudaSuccess ? 0 : 3;
}
