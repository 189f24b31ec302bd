// A C++ caller of the reference's launcher API, built against
// include/bitcache_b200_compat.cuh and linked with libbitcache_b200.so, the
// way the reference's own C++ tests and benchmarks call it
// (tests/test_correctness.cu:109-117, benchmarks/bench_latency.cu:76-79 of
// the reference): device buffers from cudaMalloc, the launch_* functions on
// the default stream, then one synchronisation.
//
// Usage: launchers_caller <dir> <batch> <n_heads> <seq_len> <head_dim>
// Reads <dir>/q.bin [B*H][D], k.bin and v.bin [B*H*S][D] (fp16) and tok.bin
// [B*H][D] (one decode token); writes the encodings, both attention outputs,
// the entropy, the precision modes and an online-encoded ring to <dir>.
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

#include "bitcache_b200_compat.cuh"

#define CHECK(x)                                                                      \
    do {                                                                              \
        cudaError_t e_ = (x);                                                         \
        if (e_ != cudaSuccess) {                                                      \
            std::fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
            return 2;                                                                 \
        }                                                                             \
    } while (0)
#define LAUNCHED(what)                                                                \
    do {                                                                              \
        if (bc_last_status() != BC_OK) {                                              \
            std::fprintf(stderr, "%s: %s\n", what, bc_status_string(bc_last_status())); \
            return 3;                                                                 \
        }                                                                             \
    } while (0)

static std::vector<char> read_file(const std::string& path) {
    std::vector<char> b;
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return b;
    std::fseek(f, 0, SEEK_END);
    b.resize(std::ftell(f));
    std::fseek(f, 0, SEEK_SET);
    if (std::fread(b.data(), 1, b.size(), f) != b.size()) b.clear();
    std::fclose(f);
    return b;
}

static bool write_file(const std::string& path, const void* dev, size_t bytes) {
    std::vector<char> h(bytes);
    if (cudaMemcpy(h.data(), dev, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) return false;
    FILE* f = std::fopen(path.c_str(), "wb");
    if (!f) return false;
    const bool ok = std::fwrite(h.data(), 1, bytes, f) == bytes;
    std::fclose(f);
    return ok;
}

template <typename T>
static T* upload(const std::vector<char>& h) {
    void* d = nullptr;
    if (cudaMalloc(&d, h.size()) != cudaSuccess) return nullptr;
    if (cudaMemcpy(d, h.data(), h.size(), cudaMemcpyHostToDevice) != cudaSuccess) return nullptr;
    return static_cast<T*>(d);
}

int main(int argc, char** argv) {
    if (argc != 6) {
        std::fprintf(stderr, "usage: %s dir batch n_heads seq_len head_dim\n", argv[0]);
        return 1;
    }
    const std::string dir = argv[1];
    const int B = std::atoi(argv[2]), H = std::atoi(argv[3]), S = std::atoi(argv[4]), D = std::atoi(argv[5]);
    const size_t n_kv = (size_t)B * H * S, n_q = (size_t)B * H;
    const std::vector<char> hq = read_file(dir + "/q.bin"), hk = read_file(dir + "/k.bin"),
                            hv = read_file(dir + "/v.bin"), ht = read_file(dir + "/tok.bin");
    if (hq.size() != n_q * D * 2 || hk.size() != n_kv * D * 2 || hv.size() != hk.size() || ht.size() != hq.size()) {
        std::fprintf(stderr, "input sizes do not match the shape\n");
        return 1;
    }
    __half *d_Q = upload<__half>(hq), *d_K = upload<__half>(hk), *d_V = upload<__half>(hv),
           *d_T = upload<__half>(ht);
    if (!d_Q || !d_K || !d_V || !d_T) return 2;

    BinaryVec *d_Kb, *d_Vb, *d_ring_b;
    ResidualVec *d_Kr, *d_Vr, *d_ring_r;
    __half *d_out_bin, *d_out_comp;
    float* d_ent;
    PrecisionMode* d_modes;
    const int ring = 8;  // online-encode ring of 8 positions per head
    CHECK(cudaMalloc(&d_Kb, n_kv * sizeof(BinaryVec)));
    CHECK(cudaMalloc(&d_Vb, n_kv * sizeof(BinaryVec)));
    CHECK(cudaMalloc(&d_Kr, n_kv * sizeof(ResidualVec)));
    CHECK(cudaMalloc(&d_Vr, n_kv * sizeof(ResidualVec)));
    CHECK(cudaMalloc(&d_out_bin, n_q * D * sizeof(__half)));
    CHECK(cudaMalloc(&d_out_comp, n_q * D * sizeof(__half)));
    CHECK(cudaMalloc(&d_ent, n_q * sizeof(float)));
    CHECK(cudaMalloc(&d_modes, n_q * sizeof(PrecisionMode)));
    CHECK(cudaMalloc(&d_ring_b, n_q * ring * sizeof(BinaryVec)));
    CHECK(cudaMalloc(&d_ring_r, n_q * ring * sizeof(ResidualVec)));
    CHECK(cudaMemset(d_ring_b, 0, n_q * ring * sizeof(BinaryVec)));
    CHECK(cudaMemset(d_ring_r, 0, n_q * ring * sizeof(ResidualVec)));

    launch_binary_encode(d_K, d_Kb, (int)n_kv, D);
    LAUNCHED("launch_binary_encode K");
    launch_binary_encode(d_V, d_Vb, (int)n_kv, D);
    LAUNCHED("launch_binary_encode V");
    launch_residual_encode(d_K, d_Kb, d_Kr, (int)n_kv, D);
    LAUNCHED("launch_residual_encode K");
    launch_residual_encode(d_V, d_Vb, d_Vr, (int)n_kv, D);
    LAUNCHED("launch_residual_encode V");
    launch_binary_attention(d_Q, d_Kb, d_Vb, d_out_bin, B, H, S, D);
    LAUNCHED("launch_binary_attention");
    launch_compensated_attention(d_Q, d_Kb, d_Kr, d_Vb, d_Vr, d_out_comp, B, H, S, D);
    LAUNCHED("launch_compensated_attention");
    launch_compute_head_entropy(d_Q, d_Kb, d_ent, B, H, S, D);
    LAUNCHED("launch_compute_head_entropy");
    launch_adaptive_select(d_ent, d_modes, B, H, 5.0f);
    LAUNCHED("launch_adaptive_select");
    // three decode tokens into the ring; the third (current_len 10) wraps to position 2
    for (int cur : {0, 1, 10}) {
        launch_online_encode_token(cur == 1 ? d_Q : d_T, d_ring_b, d_ring_r, B, H, D, cur, ring);
        LAUNCHED("launch_online_encode_token");
    }
    CHECK(cudaDeviceSynchronize());

    const struct {
        const char* name;
        const void* ptr;
        size_t bytes;
    } outs[] = {
        {"kb.bin", d_Kb, n_kv * sizeof(BinaryVec)},         {"vb.bin", d_Vb, n_kv * sizeof(BinaryVec)},
        {"kr.bin", d_Kr, n_kv * sizeof(ResidualVec)},       {"vr.bin", d_Vr, n_kv * sizeof(ResidualVec)},
        {"out_bin.bin", d_out_bin, n_q * D * 2},            {"out_comp.bin", d_out_comp, n_q * D * 2},
        {"ent.bin", d_ent, n_q * sizeof(float)},            {"modes.bin", d_modes, n_q},
        {"ring_b.bin", d_ring_b, n_q * ring * sizeof(BinaryVec)},
        {"ring_r.bin", d_ring_r, n_q * ring * sizeof(ResidualVec)},
    };
    for (const auto& o : outs)
        if (!write_file(dir + "/" + o.name, o.ptr, o.bytes)) {
            std::fprintf(stderr, "writing %s failed\n", o.name);
            return 2;
        }
    std::printf("ok\n");
    return 0;
}
