// Golden-case runner for ChunkGatedDeltaRuleFwdH through this library's C ABI.
//
// It is the counterpart of the reference's example runner
// (code/examples/test_aclnn_chunk_gated_delta_rule_fwd_h.cpp): same command
// line, same case directory, same output files, so a directory written by the
// reference's golden generator runs unchanged here.
//
//   cgdr_fwd_h_case CASE_DIR [DEVICE_ID]
//
// CASE_DIR holds
//   manifest.json               integers total_tokens, total_chunks, hv, hk, dim
//   input_k.bin                 bf16 [1, T, HK, D]
//   input_w.bin, input_u.bin    bf16 [1, HV, T, D]
//   input_g.bin                 fp32 [1, HV, T]
//   input_cu_seqlens.bin        int64 [N + 1]
//   input_chunk_indices.bin     int64 [NT, 2]
//   input_initial_state.bin     bf16 [N, HV, D, D] (optional)
// and receives actual_h.bin (bf16 [1, HV, NT, D, D]), actual_v.bin (bf16
// [1, HV, T, D]) and actual_final_state.bin (bf16 [N, HV, D, D]).  The op runs
// in the reference's layout (head-major) and arithmetic (its rounding chain),
// i.e. the plain phase-1 entry cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize.
//
// Exit codes: 0 success, 1 failure (message on stderr), 2 usage.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <initializer_list>
#include <iostream>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../include/cgdr_fwd_h.h"

namespace {

struct Failure : std::runtime_error {
    using std::runtime_error::runtime_error;
};

void cuda_ok(cudaError_t e, const char* what)
{
    if (e != cudaSuccess) throw Failure(std::string(what) + ": " + cudaGetErrorString(e));
}

void cgdr_ok(cgdrStatus st, const char* what)
{
    if (st != CGDR_STATUS_SUCCESS)
        throw Failure(std::string(what) + " returned " + std::to_string(static_cast<int>(st)) + ": " +
                      cgdrGetLastErrorMessage());
}

std::string path_join(const std::string& dir, const char* name)
{
    return dir.empty() || dir.back() == '/' ? dir + name : dir + "/" + name;
}

bool file_exists(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    return static_cast<bool>(f);
}

std::vector<char> read_file(const std::string& path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f) throw Failure("cannot open " + path);
    std::ostringstream ss;
    ss << f.rdbuf();
    const std::string s = ss.str();
    return std::vector<char>(s.begin(), s.end());
}

void write_file(const std::string& path, const std::vector<char>& data)
{
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    if (!f || !f.write(data.data(), static_cast<std::streamsize>(data.size()))) throw Failure("cannot write " + path);
}

// The integer value of "key" in a flat JSON object (enough for the manifest).
int64_t json_int(const std::string& json, const std::string& key)
{
    const std::string quoted = "\"" + key + "\"";
    size_t at = json.find(quoted);
    if (at == std::string::npos) throw Failure("manifest.json has no \"" + key + "\"");
    at = json.find(':', at + quoted.size());
    if (at == std::string::npos) throw Failure("manifest.json: no value for \"" + key + "\"");
    ++at;
    while (at < json.size() && (json[at] == ' ' || json[at] == '\t' || json[at] == '\n' || json[at] == '\r')) ++at;
    size_t end = at;
    if (end < json.size() && json[end] == '-') ++end;
    while (end < json.size() && json[end] >= '0' && json[end] <= '9') ++end;
    if (end == at) throw Failure("manifest.json: \"" + key + "\" is not an integer");
    return std::stoll(json.substr(at, end - at));
}

int64_t element_bytes(cgdrDataType dt)
{
    switch (dt) {
    case CGDR_DT_BF16:
    case CGDR_DT_FLOAT16: return 2;
    case CGDR_DT_FLOAT32:
    case CGDR_DT_INT32: return 4;
    case CGDR_DT_INT64: return 8;
    }
    return 0;
}

// A contiguous device buffer and its cgdrTensor descriptor.
struct DeviceTensor {
    cgdrTensor desc;
    size_t bytes = 0;

    DeviceTensor(std::initializer_list<int64_t> shape, cgdrDataType dt)
    {
        std::memset(&desc, 0, sizeof(desc));
        desc.dtype = dt;
        desc.ndim = static_cast<int32_t>(shape.size());
        int64_t count = 1;
        int i = 0;
        for (int64_t d : shape) {
            if (d < 0) throw Failure("negative dimension in a tensor shape");
            desc.shape[i++] = d;
            count *= d;
        }
        int64_t stride = 1;
        for (int j = desc.ndim - 1; j >= 0; --j) {
            desc.strides[j] = stride;
            stride *= desc.shape[j];
        }
        bytes = static_cast<size_t>(count * element_bytes(dt));
        if (bytes > 0) cuda_ok(cudaMalloc(&desc.data, bytes), "cudaMalloc");
    }
    ~DeviceTensor()
    {
        if (desc.data) cudaFree(desc.data);
    }
    DeviceTensor(const DeviceTensor&) = delete;
    DeviceTensor& operator=(const DeviceTensor&) = delete;

    void load(const std::string& path)
    {
        const std::vector<char> host = read_file(path);
        if (host.size() != bytes)
            throw Failure(path + " holds " + std::to_string(host.size()) + " bytes, expected " + std::to_string(bytes));
        if (bytes > 0) cuda_ok(cudaMemcpy(desc.data, host.data(), bytes, cudaMemcpyHostToDevice), "cudaMemcpy (to device)");
    }
    void save(const std::string& path) const
    {
        std::vector<char> host(bytes);
        if (bytes > 0) cuda_ok(cudaMemcpy(host.data(), desc.data, bytes, cudaMemcpyDeviceToHost), "cudaMemcpy (to host)");
        write_file(path, host);
    }
};

int run_case(const std::string& dir, int device)
{
    const std::vector<char> manifest_bytes = read_file(path_join(dir, "manifest.json"));
    const std::string manifest(manifest_bytes.begin(), manifest_bytes.end());
    const int64_t T = json_int(manifest, "total_tokens");
    const int64_t NT = json_int(manifest, "total_chunks");
    const int64_t HV = json_int(manifest, "hv");
    const int64_t HK = json_int(manifest, "hk");
    const int64_t D = json_int(manifest, "dim");

    const std::string cu_path = path_join(dir, "input_cu_seqlens.bin");
    const std::vector<char> cu_bytes = read_file(cu_path);
    if (cu_bytes.size() < 2 * sizeof(int64_t) || cu_bytes.size() % sizeof(int64_t) != 0)
        throw Failure("input_cu_seqlens.bin must hold at least two int64 values");
    const int64_t N = static_cast<int64_t>(cu_bytes.size() / sizeof(int64_t)) - 1;
    const bool has_h0 = file_exists(path_join(dir, "input_initial_state.bin"));
    std::cout << "case " << dir << ": T=" << T << " chunks=" << NT << " sequences=" << N << " hv=" << HV
              << " hk=" << HK << " dim=" << D << " initial_state=" << (has_h0 ? "yes" : "no") << std::endl;
    cuda_ok(cudaSetDevice(device), "cudaSetDevice");

    DeviceTensor k({1, T, HK, D}, CGDR_DT_BF16);
    DeviceTensor w({1, HV, T, D}, CGDR_DT_BF16);
    DeviceTensor u({1, HV, T, D}, CGDR_DT_BF16);
    DeviceTensor g({1, HV, T}, CGDR_DT_FLOAT32);
    DeviceTensor cu({N + 1}, CGDR_DT_INT64);
    DeviceTensor ci({NT, 2}, CGDR_DT_INT64);
    DeviceTensor h0({has_h0 ? N : 0, HV, D, D}, CGDR_DT_BF16);
    DeviceTensor h({1, HV, NT, D, D}, CGDR_DT_BF16);
    DeviceTensor v({1, HV, T, D}, CGDR_DT_BF16);
    DeviceTensor fin({N, HV, D, D}, CGDR_DT_BF16);
    k.load(path_join(dir, "input_k.bin"));
    w.load(path_join(dir, "input_w.bin"));
    u.load(path_join(dir, "input_u.bin"));
    g.load(path_join(dir, "input_g.bin"));
    cu.load(cu_path);
    ci.load(path_join(dir, "input_chunk_indices.bin"));
    if (has_h0) h0.load(path_join(dir, "input_initial_state.bin"));

    uint64_t ws_size = 0;
    cgdrExecutor* executor = nullptr;
    cgdr_ok(cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize(&k.desc, &w.desc, &u.desc, &g.desc,
                                                         has_h0 ? &h0.desc : nullptr, &cu.desc, &ci.desc, 64, &h.desc,
                                                         &v.desc, &fin.desc, &ws_size, &executor),
            "cgdrChunkGatedDeltaRuleFwdHGetWorkspaceSize");
    void* ws = nullptr;
    cudaError_t e = cudaMalloc(&ws, ws_size > 0 ? ws_size : 256);
    if (e != cudaSuccess) {
        cgdrDestroyExecutor(executor);
        cuda_ok(e, "cudaMalloc (workspace)");
    }
    cudaStream_t stream = nullptr;
    e = cudaStreamCreate(&stream);
    if (e != cudaSuccess) {
        cgdrDestroyExecutor(executor);
        cudaFree(ws);
        cuda_ok(e, "cudaStreamCreate");
    }
    // phase 2 consumes the executor whatever the outcome
    cgdrStatus st = cgdrChunkGatedDeltaRuleFwdH(ws, ws_size, executor, stream);
    int32_t device_status = 0;
    if (st == CGDR_STATUS_SUCCESS) st = cgdrReadDeviceStatus(ws, ws_size, stream, &device_status);
    cudaStreamDestroy(stream);
    cudaFree(ws);
    if (st == CGDR_STATUS_DEVICE_ERROR)
        throw Failure("the kernel flagged device status " + std::to_string(device_status));
    cgdr_ok(st, "cgdrChunkGatedDeltaRuleFwdH");

    h.save(path_join(dir, "actual_h.bin"));
    v.save(path_join(dir, "actual_v.bin"));
    fin.save(path_join(dir, "actual_final_state.bin"));
    std::cout << "wrote actual_h.bin, actual_v.bin and actual_final_state.bin" << std::endl;
    return 0;
}

}  // namespace

int main(int argc, char** argv)
{
    if (argc < 2 || argc > 3) {
        std::cerr << "usage: " << argv[0] << " CASE_DIR [DEVICE_ID]" << std::endl;
        return 2;
    }
    try {
        return run_case(argv[1], argc == 3 ? std::stoi(argv[2]) : 0);
    } catch (const std::exception& ex) {
        std::cerr << "error: " << ex.what() << std::endl;
        return 1;
    }
}
