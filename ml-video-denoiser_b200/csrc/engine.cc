#include "engine.h"

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <stdexcept>

#include "fused_block.h"
#include "status.h"

namespace dnb {

int launch_warp_pixel(const __half* feat, const __half* off, int off_stride, __half* out, int nimg,
                      int H, int W, int C, float sx, float sy, cudaStream_t s);
int launch_dw_pair(const __half* a, const __half* b, const float* w, __half* out, int H, int W, int C, cudaStream_t s);

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int d) {
        cudaGetDevice(&prev);
        if (prev != d) cudaSetDevice(d);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

uint32_t kmajor_offset_host(uint32_t row, uint32_t kchunk, uint32_t sbo) {
    return (row >> 3) * sbo + kchunk * 128u + (row & 7u) * 16u;
}

int next_pow2(int v) {
    int p = 1;
    while (p < v) p <<= 1;
    return p;
}
int round_up(int v, int m) { return (v + m - 1) / m * m; }
size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

struct Packer {
    std::vector<uint8_t> host;
    size_t add(const void* p, size_t bytes) {
        const size_t off = align256(host.size());
        host.resize(off + bytes);
        if (bytes) std::memcpy(host.data() + off, p, bytes);
        return off;
    }
    size_t add_f32(const std::vector<float>& v) { return add(v.data(), v.size() * sizeof(float)); }
};

// N tile of a GEMM writing n columns: up to 256 wide, which halves the
// shared-memory operand traffic per MMA against 128 (the tensor core reads
// A once per 256 output columns).
int store_nt(int n) { return std::min(256, next_pow2(std::max(16, n))); }

// Pack W[rows][K] (row-major fp32, src row per packed row, -1 = zero row)
// into the tile image the GEMM kernel bulk-copies: tiles [n_tile][k_chunk],
// each NT x KC fp16 in the no-swizzle K-major core-matrix layout (8 rows x
// 16 B per core matrix, lbo 128 B). With `ln` (gamma, beta of the LayerNorm
// that precedes the conv) the LN is folded: B = fp16(W * gamma),
// c1[n] = sum_k B[n,k], bias'[n] = bias[n] + sum_k beta[k] W[n,k].
struct LnFold {
    const std::vector<float>* gamma = nullptr;
    const std::vector<float>* beta = nullptr;
};

GemmW pack_rows(Packer& pk, const std::vector<float>& W, int K, const std::vector<int>& rows, int NT,
                const std::vector<float>* bias, int n_out, LnFold ln = {}, int seg_c = 0) {
    GemmW g;
    g.NT = NT;
    g.K = K;
    g.n_out = n_out;
    const int N = static_cast<int>(rows.size());
    // K chunk: 16 / 32 / 64 channels (one swizzled TMA box of 32 / 64 / 128 B
    // rows). A concat of narrower segments chunks at the segment width; 8-wide
    // segments use the interleaved (unswizzled) A layout.
    if (seg_c > 0 && seg_c < 64 && K > seg_c) {
        g.KC = seg_c < 16 ? 16 : seg_c;
        g.a_swz = seg_c < 16 ? 0 : 2 * g.KC;
    } else {
        g.KC = K <= 16 ? 16 : (K <= 32 ? 32 : 64);
        // A box never wider than the source: 8-channel sources stay interleaved.
        g.a_swz = K < g.KC ? 0 : 2 * g.KC;
    }
    const int Kp = round_up(K, g.KC);
    g.k_chunks = Kp / g.KC;
    g.n_tiles = (N + NT - 1) / NT;
    const uint32_t sbo = static_cast<uint32_t>(g.KC / 8) * 128u;
    const size_t tile_bytes = static_cast<size_t>(NT) * g.KC * 2;
    std::vector<uint8_t> buf(tile_bytes * g.n_tiles * g.k_chunks, 0);
    const size_t padded = static_cast<size_t>(g.n_tiles) * NT;
    std::vector<float> bvec(padded, 0.f), c1(padded, 0.f);
    for (int n = 0; n < N; ++n) {
        const int src = rows[n];
        if (src < 0) continue;
        const int t = n / NT, r = n % NT;
        double sum_b = 0.0, sum_c1 = 0.0;
        for (int kk = 0; kk < K; ++kk) {
            const float w = W[static_cast<size_t>(src) * K + kk];
            const float wg = ln.gamma ? w * (*ln.gamma)[kk] : w;
            const __half h = __float2half(wg);
            sum_c1 += static_cast<double>(__half2float(h));
            if (ln.beta) sum_b += static_cast<double>((*ln.beta)[kk]) * w;
            const int j = kk / g.KC, k = kk % g.KC;
            uint8_t* tile = buf.data() + (static_cast<size_t>(t) * g.k_chunks + j) * tile_bytes;
            std::memcpy(tile + kmajor_offset_host(r, k / 8, sbo) + (k % 8) * 2, &h, 2);
        }
        bvec[n] = (bias ? (*bias)[src] : 0.f) + static_cast<float>(sum_b);
        c1[n] = static_cast<float>(sum_c1);
    }
    g.bpack = pk.add(buf.data(), buf.size());
    if (bias || ln.beta) {
        g.bias = pk.add_f32(bvec);
        g.has_bias = true;
    }
    if (ln.gamma) {
        g.c1 = pk.add_f32(c1);
        g.has_c1 = true;
    }
    return g;
}

std::vector<int> iota_rows(int n) {
    std::vector<int> r(n);
    for (int i = 0; i < n; ++i) r[i] = i;
    return r;
}

GemmW pack_gemm(Packer& pk, const std::vector<float>& W, int N, int K, int NT, const std::vector<float>* bias,
                int n_out, LnFold ln = {}, int seg_c = 0) {
    return pack_rows(pk, W, K, iota_rows(N), NT, bias, n_out, ln, seg_c);
}

// conv4 of a NAFBlock: the two SimpleGate halves are interleaved per tile so
// that output channel c and its gate c + half land in the same tile.
GemmW pack_gate(Packer& pk, const std::vector<float>& W, const std::vector<float>& bias, int half, int K,
                LnFold ln = {}) {
    const int hnt = std::min(128, next_pow2(std::max(16, half)));
    const int NT = 2 * hnt;
    const int n_tiles = (half + hnt - 1) / hnt;
    std::vector<int> rows(static_cast<size_t>(n_tiles) * NT, -1);
    for (int t = 0; t < n_tiles; ++t)
        for (int r = 0; r < hnt; ++r) {
            const int o = t * hnt + r;
            if (o >= half) break;
            rows[t * NT + r] = o;
            rows[t * NT + hnt + r] = half + o;
        }
    return pack_rows(pk, W, K, rows, NT, &bias, half, ln);
}

std::vector<int64_t> shape_of(const HostWeights& hw, const std::string& n) { return hw.entry(n).shape; }

void expect_shape(const HostWeights& hw, const std::string& n, std::vector<int64_t> want) {
    const auto& s = hw.entry(n).shape;
    if (s != want) {
        std::string a, b;
        for (auto v : s) a += std::to_string(v) + ",";
        for (auto v : want) b += std::to_string(v) + ",";
        throw FormatError("unexpected shape for " + n + ": (" + a + ") expected (" + b + ")");
    }
}

int count_levels(const HostWeights& hw, const std::string& root) {
    int n = 0;
    while (hw.contains(root + "." + std::to_string(n) + ".0.conv1.weight")) ++n;
    return n;
}

int count_blocks(const HostWeights& hw, const std::string& root) {
    int n = 0;
    while (hw.contains(root + "." + std::to_string(n) + ".conv1.weight")) ++n;
    return n;
}

}  // namespace

// ---------------------------------------------------------------------------
// Construction: discover the architecture from the weight keys (the way the
// reference does, src/models/nafnet.cu:78-92, 281-333) and pack everything.
// ---------------------------------------------------------------------------

Engine::Engine(const std::string& manifest_path, int device) : device_(device) {
    HostWeights hw(manifest_path);
    DeviceGuard g(device_);
    build(hw);
}

Engine::~Engine() {
    DeviceGuard g(device_);
    for (auto e : prof_pool_) cudaEventDestroy(e);
    if (warena_) cudaFree(warena_);
    if (aarena_) cudaFree(aarena_);
}

void Engine::build(const HostWeights& hw) {
    Packer pk;
    const int levels = count_levels(hw, "encoders");
    if (levels <= 0) throw FormatError("NAFNet: no encoder levels found in exported weights");
    pad_multiple_ = 1 << levels;
    info_.num_levels = levels;

    const auto intro_s = shape_of(hw, "intro.weight");
    if (intro_s.size() != 4 || intro_s[2] != 3 || intro_s[3] != 3)
        throw FormatError("intro.weight must be (C0, Cin, 3, 3)");
    const int C0 = static_cast<int>(intro_s[0]);
    info_.in_channels = static_cast<int>(intro_s[1]);
    info_.base_channels = C0;
    if (C0 % 8 != 0) throw FormatError("base channel count must be a multiple of 8");
    expect_shape(hw, "intro.bias", {C0});
    expect_shape(hw, "ending.weight", {3, C0, 3, 3});
    expect_shape(hw, "ending.bias", {3});
    intro_w_ = pk.add_f32(hw.to_f32("intro.weight"));
    intro_b_ = pk.add_f32(hw.to_f32("intro.bias"));
    {
        const auto w = hw.to_f32("ending.weight");
        std::vector<float> wl(27 * C0);
        for (int o = 0; o < 3; ++o)
            for (int c = 0; c < C0; ++c)
                for (int t = 0; t < 9; ++t) wl[(o * 9 + t) * C0 + c] = w[(o * C0 + c) * 9 + t];
        ending_w_ = pk.add_f32(wl);
        ending_b_ = pk.add_f32(hw.to_f32("ending.bias"));
        if (ending_tc_supported(C0)) {
            // B tiles of the tensor-core ending: per (tap column kx, 16-channel
            // K step) three stacked taps ky = 2, 1, 0, each [16 rows x 16] with
            // output channels 0..2 in rows 0..2 (the rest zero).
            const int KS = C0 / 16;
            const size_t tap_bytes = 16 * 32;
            std::vector<uint8_t> wb(9 * KS * tap_bytes, 0);
            for (int o = 0; o < 3; ++o)
                for (int t = 0; t < 9; ++t)
                    for (int c = 0; c < C0; ++c) {
                        const __half h = __float2half(w[(o * C0 + c) * 9 + t]);
                        const int ks = c / 16, k = c % 16, ky = t / 3, kx = t % 3;
                        uint8_t* tile = wb.data() + ((static_cast<size_t>(kx) * KS + ks) * 3 + (2 - ky)) * tap_bytes;
                        std::memcpy(tile + kmajor_offset_host(o, k / 8, 256) + (k % 8) * 2, &h, 2);
                    }
            ending_tc_w_ = pk.add(wb.data(), wb.size());
        }
    }

    auto block = [&](const std::string& pre, int C) {
        BlockW b;
        b.C = C;
        const auto s1 = shape_of(hw, pre + ".conv1.weight");
        const auto s4 = shape_of(hw, pre + ".conv4.weight");
        if (s1.size() != 4 || s1[1] != C || s1[0] % 2 != 0)
            throw FormatError(pre + ".conv1.weight has an unexpected shape");
        if (s4.size() != 4 || s4[1] != C || s4[0] % 2 != 0)
            throw FormatError(pre + ".conv4.weight has an unexpected shape");
        b.dw = static_cast<int>(s1[0] / 2);
        b.ffn = static_cast<int>(s4[0] / 2);
        if (b.dw % 8 != 0 || b.ffn % 8 != 0) throw FormatError(pre + ": channel counts must be multiples of 8");
        expect_shape(hw, pre + ".norm1.weight", {C});
        expect_shape(hw, pre + ".norm1.bias", {C});
        expect_shape(hw, pre + ".norm2.weight", {C});
        expect_shape(hw, pre + ".norm2.bias", {C});
        expect_shape(hw, pre + ".beta", {1, C, 1, 1});
        expect_shape(hw, pre + ".gamma", {1, C, 1, 1});
        expect_shape(hw, pre + ".conv1.bias", {2 * b.dw});
        expect_shape(hw, pre + ".conv2.weight", {2 * b.dw, 1, 3, 3});
        expect_shape(hw, pre + ".conv2.bias", {2 * b.dw});
        expect_shape(hw, pre + ".sca.1.weight", {b.dw, b.dw, 1, 1});
        expect_shape(hw, pre + ".sca.1.bias", {b.dw});
        expect_shape(hw, pre + ".conv3.weight", {C, b.dw, 1, 1});
        expect_shape(hw, pre + ".conv3.bias", {C});
        expect_shape(hw, pre + ".conv4.bias", {2 * b.ffn});
        expect_shape(hw, pre + ".conv5.weight", {C, b.ffn, 1, 1});
        expect_shape(hw, pre + ".conv5.bias", {C});
        const auto ln1w = hw.to_f32(pre + ".norm1.weight"), ln1b = hw.to_f32(pre + ".norm1.bias");
        const auto ln2w = hw.to_f32(pre + ".norm2.weight"), ln2b = hw.to_f32(pre + ".norm2.bias");
        b.ln1w = pk.add_f32(ln1w);
        b.ln1b = pk.add_f32(ln1b);
        b.ln2w = pk.add_f32(ln2w);
        b.ln2b = pk.add_f32(ln2b);
        b.beta = pk.add_f32(hw.to_f32(pre + ".beta"));
        b.gamma = pk.add_f32(hw.to_f32(pre + ".gamma"));
        const auto b1 = hw.to_f32(pre + ".conv1.bias");
        b.conv1 = pack_gemm(pk, hw.to_f32(pre + ".conv1.weight"), 2 * b.dw, C, store_nt(2 * b.dw), &b1,
                            2 * b.dw, LnFold{&ln1w, &ln1b});
        {
            const auto w2 = hw.to_f32(pre + ".conv2.weight");
            std::vector<float> wt(9 * 2 * b.dw);
            for (int c = 0; c < 2 * b.dw; ++c)
                for (int t = 0; t < 9; ++t) wt[t * 2 * b.dw + c] = w2[c * 9 + t];
            b.dw_w = pk.add_f32(wt);
            std::vector<__half> wt16(wt.size());
            for (size_t i = 0; i < wt.size(); ++i) wt16[i] = __float2half_rn(wt[i]);
            b.dw_w16 = pk.add(wt16.data(), wt16.size() * sizeof(__half));
            b.dw_b = pk.add_f32(hw.to_f32(pre + ".conv2.bias"));
        }
        b.sca_w = pk.add_f32(hw.to_f32(pre + ".sca.1.weight"));
        b.sca_b = pk.add_f32(hw.to_f32(pre + ".sca.1.bias"));
        const auto b3 = hw.to_f32(pre + ".conv3.bias");
        b.conv3 = pack_gemm(pk, hw.to_f32(pre + ".conv3.weight"), C, b.dw, store_nt(C), &b3, C);
        b.conv4 = pack_gate(pk, hw.to_f32(pre + ".conv4.weight"), hw.to_f32(pre + ".conv4.bias"), b.ffn, C,
                            LnFold{&ln2w, &ln2b});
        const auto b5 = hw.to_f32(pre + ".conv5.bias");
        b.conv5 = pack_gemm(pk, hw.to_f32(pre + ".conv5.weight"), C, b.ffn, store_nt(C), &b5, C);
        if (deep_b_supported(C, b.dw, b.ffn)) {
            std::vector<int> rows(static_cast<size_t>(b.ffn / 64) * 128);
            for (int j = 0; j < b.ffn / 64; ++j)
                for (int r = 0; r < 64; ++r) {
                    rows[j * 128 + r] = 64 * j + r;
                    rows[j * 128 + 64 + r] = b.ffn + 64 * j + r;
                }
            const auto b4 = hw.to_f32(pre + ".conv4.bias");
            b.d4 = pack_rows(pk, hw.to_f32(pre + ".conv4.weight"), C, rows, 128, &b4, b.ffn, LnFold{&ln2w, &ln2b});
            b.deep = true;
        }
        if (fused_supported(C, b.dw, b.ffn)) {
            b.fused = true;
            const auto b4 = hw.to_f32(pre + ".conv4.bias");
            b.f1 = pack_gemm(pk, hw.to_f32(pre + ".conv1.weight"), 2 * b.dw, C, 2 * b.dw, &b1, 2 * b.dw,
                             LnFold{&ln1w, &ln1b});
            b.f3 = pack_gemm(pk, hw.to_f32(pre + ".conv3.weight"), C, b.dw, C, &b3, C);
            b.f4 = pack_gemm(pk, hw.to_f32(pre + ".conv4.weight"), 2 * b.ffn, C, 2 * b.ffn, &b4, 2 * b.ffn);
            b.f5 = pack_gemm(pk, hw.to_f32(pre + ".conv5.weight"), C, b.ffn, C, &b5, C);
        }
        if (b.fused && fused_a_tc_supported(C, b.dw)) {
            // Phase A as one 3x3 conv of the normalised input:
            // Weff[t][o][c] = dw[o][t] * W1[o][c] * gamma1[c] (fp16), packed per
            // (tap column kx, 16-channel K step) as three stacked [2dw x 16]
            // no-swizzle K-major tiles, taps ky = 2, 1, 0;
            // b1'[o] = b1[o] + sum_c beta1[c] W1[o][c] (the kernel forms the
            // depthwise bias b_dw + b1' * sum of the in-image taps' dw).
            const int N2 = 2 * b.dw, KS = C / 16;
            const auto w1 = hw.to_f32(pre + ".conv1.weight");
            const auto w2 = hw.to_f32(pre + ".conv2.weight");
            const size_t tap_bytes = static_cast<size_t>(N2) * 32;
            std::vector<uint8_t> wb(9 * KS * tap_bytes, 0);
            std::vector<float> b1p(N2);
            for (int o = 0; o < N2; ++o) {
                double sb = 0.0;
                for (int c = 0; c < C; ++c) sb += static_cast<double>(ln1b[c]) * w1[static_cast<size_t>(o) * C + c];
                b1p[o] = b1[o] + static_cast<float>(sb);
                for (int t = 0; t < 9; ++t)
                    for (int c = 0; c < C; ++c) {
                        const float v = w2[o * 9 + t] * w1[static_cast<size_t>(o) * C + c] * ln1w[c];
                        const __half h = __float2half(v);
                        const int ks = c / 16, k = c % 16, ky = t / 3, kx = t % 3;
                        // (kx, K step) tiles of three stacked taps [ky=2 | ky=1 | ky=0]
                        uint8_t* tile = wb.data() + ((static_cast<size_t>(kx) * KS + ks) * 3 + (2 - ky)) * tap_bytes;
                        std::memcpy(tile + kmajor_offset_host(o, k / 8, 256) + (k % 8) * 2, &h, 2);
                    }
            }
            b.fa_w = pk.add(wb.data(), wb.size());
            b.fa_b1 = pk.add_f32(b1p);
            b.fa_tc = true;
        }
        return b;
    };

    levels_.resize(levels);
    int C = C0;
    for (int l = 0; l < levels; ++l) {
        Level& L = levels_[l];
        L.C = C;
        info_.enc_channels.push_back(C);
        const std::string er = "encoders." + std::to_string(l);
        for (int i = 0, n = count_blocks(hw, er); i < n; ++i) L.enc.push_back(block(er + "." + std::to_string(i), C));
        // 2x2 stride-2 down: K index = tap * C + c, tap = ky*2 + kx.
        const std::string dn = "downs." + std::to_string(l) + ".body";
        expect_shape(hw, dn + ".weight", {2 * C, C, 2, 2});
        expect_shape(hw, dn + ".bias", {2 * C});
        const auto wd = hw.to_f32(dn + ".weight");
        std::vector<float> wl(static_cast<size_t>(2 * C) * 4 * C);
        for (int n = 0; n < 2 * C; ++n)
            for (int c = 0; c < C; ++c)
                for (int t = 0; t < 4; ++t) wl[static_cast<size_t>(n) * 4 * C + t * C + c] = wd[(n * C + c) * 4 + t];
        const auto bd = hw.to_f32(dn + ".bias");
        L.down = pack_gemm(pk, wl, 2 * C, 4 * C, store_nt(2 * C), &bd, 2 * C);
        C *= 2;
    }
    for (int i = 0, n = count_blocks(hw, "middle"); i < n; ++i) middle_.push_back(block("middle." + std::to_string(i), C));
    for (int d = 0; d < levels; ++d) {
        // ups.d feeds resolution level lev = levels-1-d: 1x1 C -> 2C (no bias), PixelShuffle(2).
        const int lev = levels - 1 - d;
        const int Cin = C, Cout = C / 2;
        const std::string un = "ups." + std::to_string(d) + ".body.0.weight";
        expect_shape(hw, un, {2 * Cin, Cin, 1, 1});
        const auto wu = hw.to_f32(un);
        // packed column n' = ij * Cout + c  <-  PixelShuffle source channel 4c + ij
        std::vector<float> wl(static_cast<size_t>(4 * Cout) * Cin);
        for (int ij = 0; ij < 4; ++ij)
            for (int c = 0; c < Cout; ++c)
                std::memcpy(&wl[static_cast<size_t>(ij * Cout + c) * Cin], &wu[static_cast<size_t>(4 * c + ij) * Cin],
                            Cin * sizeof(float));
        levels_[lev].up = pack_gemm(pk, wl, 4 * Cout, Cin, store_nt(4 * Cout), nullptr, 4 * Cout);
        C = Cout;
        const std::string dr = "decoders." + std::to_string(d);
        for (int i = 0, n = count_blocks(hw, dr); i < n; ++i)
            levels_[lev].dec.push_back(block(dr + "." + std::to_string(i), C));
    }

    // Temporal models.
    const bool legacy = hw.contains("temporal_mix.0.weight");
    const bool pyt = hw.contains("temporal_mix.0.0.weight");
    // NAFBlocks of a mix stage: root.1, root.2, ... (root.0 is the 1x1 conv).
    auto mix_blocks = [&](const std::string& root, int Cl) {
        std::vector<BlockW> v;
        for (int i = 1; hw.contains(root + "." + std::to_string(i) + ".conv1.weight"); ++i)
            v.push_back(block(root + "." + std::to_string(i), Cl));
        return v;
    };
    if (pyt) {
        info_.kind = 2;
        const auto& s0 = hw.entry("temporal_mix.0.0.weight").shape;
        if (s0.size() != 4 || s0[1] % C0 != 0) throw FormatError("temporal_mix.0.0.weight: unexpected shape");
        const int T = static_cast<int>(s0[1] / C0);
        if (T < 2) throw FormatError("temporal model needs num_frames >= 2");
        if (T > kMaxSeg) throw FormatError("temporal model: num_frames > 8 is not supported");
        info_.num_frames = T;
        info_.use_warp = hw.contains("offset_heads.0.0.weight") ? 1 : 0;
        const int Cd = levels_[levels - 1].C * 2;
        expect_shape(hw, "bottleneck_mix.0.weight", {Cd, static_cast<int64_t>(T) * Cd, 1, 1});
        expect_shape(hw, "bottleneck_mix.0.bias", {Cd});
        const auto bb = hw.to_f32("bottleneck_mix.0.bias");
        bneck_ = pack_gemm(pk, hw.to_f32("bottleneck_mix.0.weight"), Cd, T * Cd, store_nt(Cd), &bb, Cd, LnFold{}, Cd);
        bneck_blocks_ = mix_blocks("bottleneck_mix", Cd);
        for (int l = 0; l < levels; ++l) {
            const int Cl = levels_[l].C;
            const std::string tn = "temporal_mix." + std::to_string(l);
            expect_shape(hw, tn + ".0.weight", {Cl, static_cast<int64_t>(T) * Cl, 1, 1});
            expect_shape(hw, tn + ".0.bias", {Cl});
            const auto tb = hw.to_f32(tn + ".0.bias");
            tmix_.push_back(pack_gemm(pk, hw.to_f32(tn + ".0.weight"), Cl, T * Cl, store_nt(Cl), &tb, Cl, LnFold{}, Cl));
            tmix_blocks_.push_back(mix_blocks(tn, Cl));
            if (info_.use_warp) {
                const std::string on = "offset_heads." + std::to_string(l);
                expect_shape(hw, on + ".0.weight", {2 * Cl, 1, 3, 3});
                expect_shape(hw, on + ".1.weight", {Cl, 2 * Cl, 1, 1});
                expect_shape(hw, on + ".3.weight", {2, Cl, 1, 1});
                expect_shape(hw, on + ".3.bias", {2});
                const auto w0 = hw.to_f32(on + ".0.weight");
                std::vector<float> wt(9 * 2 * Cl);
                for (int c = 0; c < 2 * Cl; ++c)
                    for (int t = 0; t < 9; ++t) wt[t * 2 * Cl + c] = w0[c * 9 + t];
                oh_dw_.push_back(pk.add_f32(wt));
                oh_pw1_.push_back(pack_gemm(pk, hw.to_f32(on + ".1.weight"), Cl, 2 * Cl, store_nt(Cl), nullptr, Cl));
                const auto b3 = hw.to_f32(on + ".3.bias");
                // 2 outputs padded to an 8-channel row (dx, dy, 0 x 6).
                oh_pw2_.push_back(pack_gemm(pk, hw.to_f32(on + ".3.weight"), 2, Cl, 16, &b3, 8));
            }
        }
    } else if (legacy) {
        info_.kind = 1;
        const int T = hw.arch().num_frames > 0 ? hw.arch().num_frames : 3;
        if (T < 2) throw FormatError("temporal model needs num_frames >= 2");
        if (T > kMaxSeg) throw FormatError("temporal model: num_frames > 8 is not supported");
        info_.num_frames = T;
        info_.use_warp = hw.contains("offset_heads.0.weight") ? 1 : 0;
        for (int l = 0; l < levels; ++l) {
            const int Cl = levels_[l].C;
            const std::string tn = "temporal_mix." + std::to_string(l);
            expect_shape(hw, tn + ".weight", {Cl, 2 * Cl, 1, 1});
            expect_shape(hw, tn + ".bias", {Cl});
            const auto w = hw.to_f32(tn + ".weight");
            // concat(ref, mean_t nbr_t) @ W^T == [ref, nbr_1..nbr_{T-1}] @ [W_ref, W_mean/(T-1), ...]^T
            std::vector<float> wl(static_cast<size_t>(Cl) * T * Cl);
            const float inv = 1.0f / static_cast<float>(T - 1);
            for (int o = 0; o < Cl; ++o)
                for (int c = 0; c < Cl; ++c) {
                    wl[static_cast<size_t>(o) * T * Cl + c] = w[static_cast<size_t>(o) * 2 * Cl + c];
                    for (int s = 1; s < T; ++s)
                        wl[static_cast<size_t>(o) * T * Cl + s * Cl + c] = w[static_cast<size_t>(o) * 2 * Cl + Cl + c] * inv;
                }
            const auto tb = hw.to_f32(tn + ".bias");
            tmix_.push_back(pack_gemm(pk, wl, Cl, T * Cl, store_nt(Cl), &tb, Cl, LnFold{}, Cl));
            if (info_.use_warp) {
                const std::string on = "offset_heads." + std::to_string(l);
                expect_shape(hw, on + ".weight", {2, 2 * Cl, 1, 1});
                expect_shape(hw, on + ".bias", {2});
                const auto ob = hw.to_f32(on + ".bias");
                // 2 outputs padded to an 8-channel row (dx, dy, 0 x 6).
                offset_heads_.push_back(pack_gemm(pk, hw.to_f32(on + ".weight"), 2, 2 * Cl, 16, &ob, 8, LnFold{}, Cl));
            }
        }
    } else if (hw.arch().type == "nafnet_temporal") {
        throw FormatError("manifest says nafnet_temporal but has no temporal_mix weights");
    }

    warena_bytes_ = align256(pk.host.size());
    cudaError_t e = cudaMalloc(&warena_, warena_bytes_);
    if (e != cudaSuccess) throw std::runtime_error(std::string("weight arena: ") + cudaGetErrorString(e));
    e = cudaMemcpy(warena_, pk.host.data(), pk.host.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) throw std::runtime_error(std::string("weight upload: ") + cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// Activation planning
// ---------------------------------------------------------------------------

void Engine::plan(const Shape& s) {
    if (aarena_ && shape_ == s) return;
    if (aarena_) {
        cudaFree(aarena_);
        aarena_ = nullptr;
    }
    shape_ = s;
    const int L = info_.num_levels;
    const bool temporal = info_.kind != 0;
    const size_t n_enc = temporal ? s.T : s.N;  // images through the encoder
    const size_t n_dec = temporal ? 1 : s.N;
    std::vector<std::pair<size_t, void**>> req;
    enc_x_.assign(L, nullptr);
    dec_x_.assign(L, nullptr);
    fused_skip_.assign(L, nullptr);
    size_t u = 0, g = 0, y = 0, t = 0, dmax = 8;
    dw_blocks_max_ = 1;
    auto account = [&](const std::vector<BlockW>& bl, size_t nimg, int h, int w) {
        const size_t hw = static_cast<size_t>(h) * w;
        for (const auto& b : bl) {
            u = std::max(u, nimg * hw * 2 * b.dw);
            g = std::max(g, nimg * hw * b.dw);
            y = std::max(y, nimg * hw * b.C);
            t = std::max(t, nimg * hw * b.ffn);
            dmax = std::max(dmax, static_cast<size_t>(b.dw));
            dw_blocks_max_ = std::max(dw_blocks_max_, dw_blocks_per_img(h, w, b.dw));
            dw_blocks_max_ = std::max(dw_blocks_max_, dw_tile_blocks_per_img(h, w));
            if (b.fused) dw_blocks_max_ = std::max(dw_blocks_max_, fused_a_grid(b.C, b.dw, static_cast<int>(nimg), h, w));
            if (b.fa_tc) dw_blocks_max_ = std::max(dw_blocks_max_, fused_a_tc_grid(b.C, static_cast<int>(nimg), h, w));
        }
    };
    for (int l = 0; l < L; ++l) {
        const int h = s.Hp >> l, w = s.Wp >> l, C = levels_[l].C;
        const size_t hw = static_cast<size_t>(h) * w;
        req.push_back({n_enc * hw * C * 2, reinterpret_cast<void**>(&enc_x_[l])});
        req.push_back({n_dec * hw * C * 2, reinterpret_cast<void**>(&dec_x_[l])});
        if (temporal) req.push_back({hw * C * 2, reinterpret_cast<void**>(&fused_skip_[l])});
        account(levels_[l].enc, n_enc, h, w);
        account(levels_[l].dec, n_dec, h, w);
    }
    const int hm = s.Hp >> L, wm = s.Wp >> L;
    const size_t hwm = static_cast<size_t>(hm) * wm;
    const int Cm = levels_[L - 1].C * 2;
    req.push_back({n_enc * hwm * Cm * 2, reinterpret_cast<void**>(&mid_x_)});
    account(middle_, 1 * (temporal ? 1 : n_enc), hm, wm);
    if (info_.kind == 2) {
        account(bneck_blocks_, 1, hm, wm);
        for (int l = 0; l < L; ++l) account(tmix_blocks_[l], 1, s.Hp >> l, s.Wp >> l);
    }
    req.push_back({u * 2, reinterpret_cast<void**>(&buf_u_)});
    req.push_back({g * 2, reinterpret_cast<void**>(&buf_g_)});
    req.push_back({y * 2, reinterpret_cast<void**>(&buf_y_)});
    req.push_back({t * 2, reinterpret_cast<void**>(&buf_t_)});
    if (temporal) {
        const size_t hw0 = static_cast<size_t>(s.Hp) * s.Wp;
        req.push_back({static_cast<size_t>(s.T) * hw0 * levels_[0].C * 2, reinterpret_cast<void**>(&warp_buf_)});
        req.push_back({hw0 * 8 * 2, reinterpret_cast<void**>(&offset_buf_)});
    }
    if (temporal) req.push_back({hwm * Cm * 2, reinterpret_cast<void**>(&bneck_x_)});
    if (info_.kind == 2) {
        if (info_.use_warp) {
            const size_t hw0 = static_cast<size_t>(s.Hp) * s.Wp;
            req.push_back({hw0 * 2 * levels_[0].C * 2, reinterpret_cast<void**>(&oh_d_)});
            req.push_back({hw0 * levels_[0].C * 2, reinterpret_cast<void**>(&oh_h_)});
        }
    }
    req.push_back({n_enc * dw_blocks_max_ * dmax * 4, reinterpret_cast<void**>(&partials_)});
    req.push_back({n_enc * 4, reinterpret_cast<void**>(&counters_)});
    req.push_back({n_enc * dmax * 4, reinterpret_cast<void**>(&sca_s_)});
    {
        size_t b3 = 0;
        auto acc_b3 = [&](const std::vector<BlockW>& bl) {
            for (const auto& b : bl)
                b3 = std::max(b3, static_cast<size_t>(b.conv3.n_tiles) * b.conv3.k_chunks * b.conv3.NT * b.conv3.KC * 2);
        };
        for (int l = 0; l < L; ++l) {
            acc_b3(levels_[l].enc);
            acc_b3(levels_[l].dec);
        }
        acc_b3(middle_);
        acc_b3(bneck_blocks_);
        for (const auto& tb : tmix_blocks_) acc_b3(tb);
        req.push_back({b3, reinterpret_cast<void**>(&b3s_)});
    }
    req.push_back({256, reinterpret_cast<void**>(&err_)});
    size_t total = 0;
    for (auto& r : req) total = align256(total) + align256(r.first);
    cudaError_t e = cudaMalloc(&aarena_, total);
    if (e != cudaSuccess) throw std::runtime_error(std::string("activation arena: ") + cudaGetErrorString(e));
    aarena_bytes_ = total;
    size_t off = 0;
    for (auto& r : req) {
        off = align256(off);
        *r.second = aarena_ + off;
        off += align256(r.first);
    }
    e = cudaMemset(counters_, 0, n_enc * 4);
    if (e == cudaSuccess) e = cudaMemset(err_, 0, 256);
    if (e != cudaSuccess) throw std::runtime_error(std::string("arena init: ") + cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------

void Engine::prof_begin(const char* kind, double bytes, double flops, cudaStream_t s) {
    if (!profiling_) return;
    while (prof_pool_.size() < prof_used_ + 2) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        prof_pool_.push_back(e);
    }
    std::string key = kind;
    if (prof_detail_ && !prof_tag_.empty()) key += "@" + prof_tag_;
    ProfRec r{key, bytes, flops, prof_pool_[prof_used_], prof_pool_[prof_used_ + 1]};
    prof_used_ += 2;
    cudaEventRecord(r.a, s);
    prof_.push_back(r);
}

void Engine::prof_end(cudaStream_t s) {
    if (!profiling_ || prof_.empty()) return;
    cudaEventRecord(prof_.back().b, s);
}

std::string Engine::profile_report() {
    DeviceGuard dg(device_);
    cudaDeviceSynchronize();
    struct Agg {
        int n = 0;
        double ms = 0, bytes = 0, flops = 0;
    };
    std::vector<std::pair<std::string, Agg>> agg;
    for (const auto& r : prof_) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, r.a, r.b);
        auto it = std::find_if(agg.begin(), agg.end(), [&](const auto& x) { return x.first == r.kind; });
        if (it == agg.end()) {
            agg.push_back({r.kind, Agg{}});
            it = agg.end() - 1;
        }
        it->second.n += 1;
        it->second.ms += ms;
        it->second.bytes += r.bytes;
        it->second.flops += r.flops;
    }
    prof_.clear();
    prof_used_ = 0;
    std::string out = "{";
    for (size_t i = 0; i < agg.size(); ++i) {
        char buf[256];
        std::snprintf(buf, sizeof(buf), "%s\"%s\": {\"launches\": %d, \"ms\": %.6f, \"bytes\": %.0f, \"flops\": %.0f}",
                      i ? ", " : "", agg[i].first.c_str(), agg[i].second.n, agg[i].second.ms, agg[i].second.bytes,
                      agg[i].second.flops);
        out += buf;
    }
    return out + "}";
}

int Engine::gemm(const GemmW& g, int pro, int epi, int amode, GemmParams p, cudaStream_t s,
                 const uint8_t* bpack_override) {
    p.bpack = bpack_override ? bpack_override : wptr<uint8_t>(g.bpack);
    p.n_tiles = g.n_tiles;
    p.k_chunks = g.k_chunks;
    p.KC = g.KC;
    p.a_swz = g.a_swz;
    p.K = g.K;
    p.bias = g.has_bias ? wptr<float>(g.bias) : nullptr;
    p.ln_c1 = g.has_c1 ? wptr<float>(g.c1) : nullptr;
    p.n_out = g.n_out;
    p.err = err_;
    // 1x1 convs with 128/256-wide tiles run on CTA pairs (cta_group::2):
    // each SM then loads half of every B tile.
    if (amode == kARows && gemm_pair_enabled_ && (g.NT == 128 || g.NT == 256) && p.nseg == 1 &&
        p.M >= 2 * 128 && (epi == kEpiStore || epi == kEpiGate || epi == kEpiResidual))
        amode = kARowsPair;
    ++launches_;
    if (profiling_) {
        const char* kind = (epi == kEpiShuffleAdd || epi == kEpiShuffleRows) ? "gemm_up_shuffle"
                           : (amode == kAS2x2 || amode == kAPairs) ? "gemm_down_s2"
                           : epi == kEpiGate     ? "gemm_ln_gate"
                           : pro == kProLayerNorm ? "gemm_ln"
                           : pro == kProScale    ? "gemm_sca_residual"
                           : epi == kEpiResidual ? "gemm_residual"
                                                 : "gemm_store";
        const double rows = p.M, n_w = static_cast<double>(g.n_tiles) * g.NT;
        double bytes = rows * g.K * 2 + n_w * g.K * 2;
        const bool shuffle = epi == kEpiShuffleAdd || epi == kEpiShuffleRows;
        const double n_out = shuffle ? 4.0 * p.out_c : p.n_out;
        bytes += rows * n_out * 2 * (epi == kEpiResidual || shuffle ? 2 : 1);
        const std::string block_tag = prof_tag_;
        if (prof_detail_)
            prof_tag_ = "M" + std::to_string(p.M) + "_N" + std::to_string(g.n_tiles * g.NT) + "_K" + std::to_string(g.K);
        prof_begin(kind, bytes, 2.0 * rows * n_w * g.K, s);
        prof_tag_ = block_tag;
    }
    const int rc = launch_gemm(p, pro, epi, amode, g.NT, s);
    launches_ += gemm_last_launches() - 1;
    prof_end(s);
    return rc;
}

// The deep second-pass kernel reads the GEMM tile images directly: conv3 and
// conv5 as single N tiles of K chunk 64, conv4 as 256-row tiles (two
// 128-channel gate halves) of K chunk 64.
static bool deep_b_layout_ok(const BlockW& b) {
    return b.deep && b.conv3.n_tiles == 1 && b.conv3.NT == b.C && b.conv3.KC == 64 && b.conv3.k_chunks * 64 == b.dw &&
           b.d4.NT == 128 && b.d4.KC == 64 && b.d4.n_tiles * 64 == b.ffn && b.d4.k_chunks * 64 == b.C &&
           b.d4.has_c1 && b.d4.has_bias && b.conv5.n_tiles == 1 && b.conv5.NT == b.C && b.conv5.KC == 64 &&
           b.conv5.k_chunks * 64 == b.ffn && b.conv3.has_bias && b.conv5.has_bias;
}

static GemmParams rows_params(int nimg, int h, int w) {
    GemmParams p{};
    p.M = nimg * h * w;
    p.hw = h * w;
    p.Ho = h;
    p.Wo = w;
    p.nseg = 1;
    return p;
}

// NAFBlock (training/models.py:166-185, src/models/nafnet.cu:146-215), in place on x.
int Engine::run_block(const BlockW& b, __half* x, int nimg, int h, int w, cudaStream_t s) {
    if (prof_detail_) prof_tag_ = "C" + std::to_string(b.C) + "_" + std::to_string(h) + "x" + std::to_string(w);
    const long long hw = static_cast<long long>(h) * w;
    if (b.fused && fused_enabled_ && nimg <= 8) {
        // Pass A: LN1 + conv1 + DW3x3 + SimpleGate + pool partials.
        FusedAParams fa{};
        fa.x = x;
        fa.g = buf_g_;
        fa.N = nimg;
        fa.H = h;
        fa.W = w;
        fa.w1 = wptr<uint8_t>(b.f1.bpack);
        fa.c1 = wptr<float>(b.f1.c1);
        fa.c2 = wptr<float>(b.f1.bias);
        fa.dw_w = wptr<float>(b.dw_w);
        fa.dw_b = wptr<float>(b.dw_b);
        fa.partials = partials_;
        fa.err = err_;
        const bool split = fa_split_enabled_ && b.fa_tc && fused_a_split_supported(b.C, b.dw, nimg);
        const bool tc = b.fa_tc && fa_tc_enabled_;
        // One image through the tensor-core pass A (either form): its last CTA
        // also runs the SCA and folds the scale into conv3's B (no SCA launch).
        const bool sca_in_a = (tc || split) && nimg == 1 && b3s_ != nullptr && b.f3.n_tiles == 1 &&
                              b.f3.k_chunks == 1 && b.f3.KC == b.dw;
        if (tc) {
            fa.weff = wptr<uint8_t>(b.fa_w);
            fa.b1p = wptr<float>(b.fa_b1);
        }
        if (sca_in_a) {
            fa.counter = counters_;
            fa.sca_w = wptr<float>(b.sca_w);
            fa.sca_b = wptr<float>(b.sca_b);
            fa.b3_src = wptr<uint8_t>(b.f3.bpack);
            fa.b3_dst = b3s_;
        }
        const int grid = split ? fused_a_split_grid(b.C, h, w)
                               : (tc ? fused_a_tc_grid(b.C, nimg, h, w) : fused_a_grid(b.C, b.dw, nimg, h, w));
        launches_ += sca_in_a ? 2 : 3;
        prof_begin("fused_block_a", static_cast<double>(nimg) * hw * (b.C + b.dw) * 2,
                   2.0 * nimg * hw * (b.C * 2 * b.dw + 2 * b.dw * 9), s);
        DN_TRY(split ? launch_fused_a_split(fa, b.C, b.dw, grid, s)
                     : (tc ? launch_fused_a_tc(fa, b.C, b.dw, grid, s) : launch_fused_a(fa, b.C, b.dw, grid, s)));
        prof_end(s);
        DwParams d{};
        d.N = nimg;
        d.H = h;
        d.W = w;
        d.D = b.dw;
        d.partials = partials_;
        d.sca_w = wptr<float>(b.sca_w);
        d.sca_b = wptr<float>(b.sca_b);
        d.s_out = sca_s_;
        // Single image: the SCA kernel writes conv3's B with the scale folded
        // in, and pass B skips its per-tile scaling of g.
        const bool fold_sca = nimg == 1 && b3s_ != nullptr;
        if (fold_sca) {
            d.bsrc = wptr<uint8_t>(b.f3.bpack);
            d.bdst = b3s_;
            d.b_rows = b.C;
            d.b_nt = b.f3.NT;
            d.b_kc = b.f3.KC;
            d.b_kchunks = b.f3.k_chunks;
        }
        if (!sca_in_a) {
            prof_begin("sca", 4.0 * nimg * grid * b.dw, 2.0 * nimg * b.dw * b.dw, s);
            DN_TRY(launch_sca(d, grid, s));
            prof_end(s);
        }
        // Pass B: SCA scale + conv3 + beta residual + LN2 + conv4 + gate + conv5 + gamma residual.
        FusedBParams fb{};
        fb.g = buf_g_;
        fb.x = x;
        fb.out = x;
        fb.M = static_cast<int>(nimg * hw);
        fb.hw = static_cast<int>(hw);
        fb.s = fold_sca ? nullptr : sca_s_;
        fb.w3 = fold_sca ? b3s_ : wptr<uint8_t>(b.f3.bpack);
        fb.w4 = wptr<uint8_t>(b.f4.bpack);
        fb.w5 = wptr<uint8_t>(b.f5.bpack);
        fb.b3 = wptr<float>(b.f3.bias);
        fb.beta = wptr<float>(b.beta);
        fb.ln_w = wptr<float>(b.ln2w);
        fb.ln_b = wptr<float>(b.ln2b);
        fb.b4 = wptr<float>(b.f4.bias);
        fb.b5 = wptr<float>(b.f5.bias);
        fb.gamma = wptr<float>(b.gamma);
        fb.err = err_;
        prof_begin("fused_block_b", static_cast<double>(nimg) * hw * (b.dw + 2 * b.C) * 2,
                   2.0 * nimg * hw * (b.dw * b.C + b.C * 2 * b.ffn + b.ffn * b.C), s);
        DN_TRY(launch_fused_b(fb, b.C, b.dw, b.ffn, s));
        prof_end(s);
        return DN_OK;
    }
    // u = conv1(LN1(x)) + b1
    GemmParams p = rows_params(nimg, h, w);
    p.seg_c = b.C;
    p.a_img_stride = hw * b.C;
    p.a[0] = x;
    p.out = buf_u_;
    p.out_c = 2 * b.dw;
    DN_TRY(gemm(b.conv1, kProLayerNorm, kEpiStore, kARows, p, s));
    // g = SG(dw3x3(u) + b2); s = W_sca * mean(g) + b_sca
    DwParams d{};
    d.u = buf_u_;
    d.g = buf_g_;
    d.w = wptr<float>(b.dw_w);
    d.w16 = wptr<__half>(b.dw_w16);
    d.b = wptr<float>(b.dw_b);
    d.N = nimg;
    d.H = h;
    d.W = w;
    d.D = b.dw;
    d.partials = partials_;
    d.counter = counters_;
    d.sca_w = wptr<float>(b.sca_w);
    d.sca_b = wptr<float>(b.sca_b);
    d.s_out = sca_s_;
    d.err = err_;
    // Single image: the SCA kernel also writes conv3's B with s folded in,
    // so conv3 needs no in-place scaling of A.
    const bool fold_sca = fused_enabled_ && nimg == 1 && b3s_ != nullptr;
    if (fold_sca) {
        d.bsrc = wptr<uint8_t>(b.conv3.bpack);
        d.bdst = b3s_;
        d.b_rows = b.C;
        d.b_nt = b.conv3.NT;
        d.b_kc = b.conv3.KC;
        d.b_kchunks = b.conv3.k_chunks;
    }
    launches_ += 2;  // depthwise + SCA
    if (fused_enabled_ && dw_tile_supported(b.dw)) {
        prof_begin("dw_tile_sca", static_cast<double>(nimg) * hw * 3 * b.dw * 2,
                   static_cast<double>(nimg) * hw * 2 * b.dw * 9 * 2 + 2.0 * b.dw * b.dw, s);
        DN_TRY(launch_dw_tile(d, s));
    } else {
        prof_begin("dw_gate_sca", static_cast<double>(nimg) * hw * 3 * b.dw * 2,
                   static_cast<double>(nimg) * hw * 2 * b.dw * 9 * 2 + 2.0 * b.dw * b.dw, s);
        DN_TRY(launch_dw_gate_sca(d, dw_blocks_per_img(h, w, b.dw), s));
    }
    prof_end(s);
    if (fold_sca && deep_b_supported(b.C, b.dw, b.ffn) && deep_b_layout_ok(b)) {
        // conv3 + beta residual + LN2 + conv4 + gate + conv5 + gamma residual
        // in one kernel; y and the gated tensor stay on chip.
        DeepBParams q{};
        q.g = buf_g_;
        q.x = x;
        q.out = x;
        q.M = static_cast<int>(hw);
        q.w3 = b3s_;
        q.w4 = wptr<uint8_t>(b.d4.bpack);
        q.w5 = wptr<uint8_t>(b.conv5.bpack);
        q.b3 = wptr<float>(b.conv3.bias);
        q.beta = wptr<float>(b.beta);
        q.c1 = wptr<float>(b.d4.c1);
        q.c2 = wptr<float>(b.d4.bias);
        q.b5 = wptr<float>(b.conv5.bias);
        q.gamma = wptr<float>(b.gamma);
        q.err = err_;
        ++launches_;
        prof_begin("deep_block_b", static_cast<double>(hw) * (b.dw + 2 * b.C) * 2,
                   2.0 * hw * (b.dw * b.C + b.C * 2 * b.ffn + b.ffn * b.C), s);
        DN_TRY(launch_deep_b(q, b.C, b.dw, b.ffn, s));
        prof_end(s);
        return DN_OK;
    }
    // y = x + beta * (conv3(g * s) + b3)
    p = rows_params(nimg, h, w);
    p.seg_c = b.dw;
    p.a_img_stride = hw * b.dw;
    p.a[0] = buf_g_;
    p.pro_scale = sca_s_;
    p.out = buf_y_;
    p.out_c = b.C;
    p.res = x;
    p.res_scale = wptr<float>(b.beta);
    if (fold_sca)
        DN_TRY(gemm(b.conv3, kProNone, kEpiResidual, kARows, p, s, b3s_));  // s folded into B by the SCA kernel
    else
        DN_TRY(gemm(b.conv3, kProScale, kEpiResidual, kARows, p, s));
    // t = SG(conv4(LN2(y)) + b4)
    p = rows_params(nimg, h, w);
    p.seg_c = b.C;
    p.a_img_stride = hw * b.C;
    p.a[0] = buf_y_;
    p.out = buf_t_;
    p.out_c = b.ffn;
    DN_TRY(gemm(b.conv4, kProLayerNorm, kEpiGate, kARows, p, s));
    // x = y + gamma * (conv5(t) + b5)
    p = rows_params(nimg, h, w);
    p.seg_c = b.ffn;
    p.a_img_stride = hw * b.ffn;
    p.a[0] = buf_t_;
    p.out = x;
    p.out_c = b.C;
    p.res = buf_y_;
    p.res_scale = wptr<float>(b.gamma);
    DN_TRY(gemm(b.conv5, kProNone, kEpiResidual, kARows, p, s));
    return DN_OK;
}

int Engine::run_stage(const std::vector<BlockW>& blocks, __half* x, int nimg, int h, int w, cudaStream_t s) {
    for (const auto& b : blocks) DN_TRY(run_block(b, x, nimg, h, w, s));
    return DN_OK;
}

// Shape of an input of N images (clips of T frames) of C x H x W, padded to
// the model's multiple; DN_OK or an error for shapes the engine rejects.
int Engine::make_shape(int N, int T, int C, int H, int W, Shape& sh) {
    if (N <= 0 || H <= 0 || W <= 0) return dn_fail(DN_ERR_INVALID_ARG, "forward: empty input");
    if (C < info_.in_channels)
        return dn_fail(DN_ERR_INVALID_ARG, "forward: input has fewer channels than model expects");
    if (C < 3) return dn_fail(DN_ERR_INVALID_ARG, "forward: expected at least 3 input channels");
    const int m = pad_multiple_;
    // Temporal models process one clip at a time: the arena (and with it the
    // frame cache of encode_frame) does not depend on N.
    sh.N = info_.kind != 0 ? 1 : N;
    sh.T = T;
    sh.H = H;
    sh.W = W;
    sh.Hp = (H + m - 1) / m * m;
    sh.Wp = (W + m - 1) / m * m;
    if (sh.Hp - H >= H || sh.Wp - W >= W)
        return dn_fail(DN_ERR_INVALID_ARG, "forward: frame smaller than the reflect padding it needs");
    if (static_cast<long long>(N) * T * sh.Hp * sh.Wp > (1LL << 30))
        return dn_fail(DN_ERR_UNSUPPORTED, "forward: input too large");
    try {
        plan(sh);
    } catch (const std::exception& e) {
        return dn_fail(DN_ERR_CUDA, e.what());
    }
    return DN_OK;
}

// Intro + encoder over `nimg` NCHW images (image stride in_stride) into
// encoder slots slot0 .. slot0 + nimg - 1: the per-level features land in
// enc_x_[l] + slot * plane_l and the deep features in mid_x_ + slot * mplane.
int Engine::encode_into(const __half* src, int nimg, int in_stride, int slot0, cudaStream_t s) {
    const Shape& sh = shape_;
    const int L = info_.num_levels;
    const int C0 = info_.base_channels;
    const int in_c = info_.in_channels;
    const int H = sh.H, W = sh.W;
    auto slot_ptr = [&](__half* base, int l) {
        const size_t plane = static_cast<size_t>(sh.Hp >> l) * (sh.Wp >> l) * (l < L ? levels_[l].C : levels_[L - 1].C * 2);
        return base + static_cast<size_t>(slot0) * plane;
    };
    IntroParams ip{};
    ip.x = src;
    ip.N = nimg;
    ip.Cin = in_c;
    ip.H = H;
    ip.W = W;
    ip.Hp = sh.Hp;
    ip.Wp = sh.Wp;
    ip.C0 = C0;
    ip.in_batch_stride = in_stride;
    ip.w = wptr<float>(intro_w_);
    ip.b = wptr<float>(intro_b_);
    ip.y = slot_ptr(enc_x_[0], 0);
    ip.err = err_;
    ++launches_;
    if (prof_detail_) prof_tag_ = "C" + std::to_string(C0) + "_" + std::to_string(sh.Hp) + "x" + std::to_string(sh.Wp);
    prof_begin("intro", static_cast<double>(nimg) * (static_cast<double>(in_c) * H * W + static_cast<double>(sh.Hp) * sh.Wp * C0) * 2,
               2.0 * nimg * sh.Hp * sh.Wp * C0 * in_c * 9, s);
    DN_TRY(fa_tc_enabled_ && intro_tc_supported(in_c, C0) ? launch_intro_tc(ip, s) : launch_intro(ip, s));
    prof_end(s);
    for (int l = 0; l < L; ++l) {
        const int h = sh.Hp >> l, w = sh.Wp >> l;
        __half* xl = slot_ptr(enc_x_[l], l);
        DN_TRY(run_stage(levels_[l].enc, xl, nimg, h, w, s));
        GemmParams p = rows_params(nimg, h / 2, w / 2);
        p.seg_c = levels_[l].C;
        p.a_img_stride = static_cast<long long>(h) * w * levels_[l].C;
        p.a[0] = xl;
        p.out = (l + 1 < L) ? slot_ptr(enc_x_[l + 1], l + 1) : slot_ptr(mid_x_, L);
        p.out_c = 2 * levels_[l].C;
        // Stride-2 A tiles by TMA (input rows viewed as pixel pairs) when a K
        // chunk fits a pair of pixels; the cp.async gather otherwise.
        const GemmW& gd = levels_[l].down;
        const bool pairs = gemm_tma_enabled_ && gd.KC <= 2 * levels_[l].C && (2 * levels_[l].C) % gd.KC == 0 &&
                           gd.a_swz == 2 * gd.KC;
        DN_TRY(gemm(gd, kProNone, kEpiStore, pairs ? kAPairs : kAS2x2, p, s));
    }
    return DN_OK;
}

// Middle + decoder + ending on `nimg` images from the deep features xm (in
// place) and the per-level skips; out = beauty + residual, NCHW.
int Engine::decode_from(__half* xm, int nimg, const std::vector<__half*>& skips, const __half* beauty,
                        int beauty_stride, __half* out, cudaStream_t s) {
    const Shape& sh = shape_;
    const int L = info_.num_levels;
    const int C0 = info_.base_channels;
    const int H = sh.H, W = sh.W;
    const int hm = sh.Hp >> L, wm = sh.Wp >> L;
    DN_TRY(run_stage(middle_, xm, nimg, hm, wm, s));
    const __half* cur = xm;
    for (int d = 0; d < L; ++d) {
        const int lev = L - 1 - d;
        const int h = sh.Hp >> (lev + 1), w = sh.Wp >> (lev + 1);
        const int Cin = levels_[lev].C * 2;
        GemmParams p = rows_params(nimg, h, w);
        p.seg_c = Cin;
        p.a_img_stride = static_cast<long long>(h) * w * Cin;
        p.a[0] = cur;
        p.out = dec_x_[lev];
        p.out_c = levels_[lev].C;
        p.skip = skips[lev];
        // PixelShuffle through a staged tile (two contiguous fine-row runs by
        // TMA) when one N tile holds all four sub-pixels of 32/64 channels.
        const GemmW& gu = levels_[lev].up;
        const bool rows = gemm_tma_enabled_ && gu.n_tiles == 1 && gu.NT == 4 * p.out_c &&
                          (p.out_c == 32 || p.out_c == 64);
        DN_TRY(gemm(gu, kProNone, rows ? kEpiShuffleRows : kEpiShuffleAdd, kARows, p, s));
        DN_TRY(run_stage(levels_[lev].dec, dec_x_[lev], nimg, 2 * h, 2 * w, s));
        cur = dec_x_[lev];
    }
    EndingParams ep{};
    ep.x = dec_x_[0];
    ep.N = nimg;
    ep.Hp = sh.Hp;
    ep.Wp = sh.Wp;
    ep.C0 = C0;
    ep.H = H;
    ep.W = W;
    ep.w = wptr<float>(ending_w_);
    ep.b = wptr<float>(ending_b_);
    ep.beauty = beauty;
    ep.beauty_batch_stride = beauty_stride;
    ep.y = out;
    ep.weff = (ending_tc_w_ && fa_tc_enabled_) ? wptr<uint8_t>(ending_tc_w_) : nullptr;
    ep.err = err_;
    ++launches_;
    prof_begin("ending", static_cast<double>(nimg) * (static_cast<double>(sh.Hp) * sh.Wp * C0 + 6.0 * H * W) * 2,
               2.0 * nimg * H * W * 3 * C0 * 9, s);
    const int rc_end = launch_ending(ep, s);
    prof_end(s);
    return rc_end;
}

// Temporal tail of one clip whose frame t sits in encoder slot slots[t]:
// the temporal fusion of the skips (and, in the PyTorch design, of the deep
// features), middle, decoder and ending; beauty = the reference frame. The
// slots are only read, so they can be reused for the next window.
int Engine::temporal_tail(const int* slots, const __half* beauty, int beauty_stride, __half* y, cudaStream_t s) {
    const Shape& sh = shape_;
    const int L = info_.num_levels;
    const int T = info_.num_frames;
    const int ref = T / 2;
    const int hm = sh.Hp >> L, wm = sh.Wp >> L;
    const size_t mplane = static_cast<size_t>(hm) * wm * levels_[L - 1].C * 2;
    if (info_.kind == 2) {
        // PyTorch NAFNetTemporal (training/models.py:738-808): bottleneck_mix
        // over the T deep features, middle, per level temporal_mix over the T
        // skips (neighbours warped by their offset head when present).
        GemmParams p = rows_params(1, hm, wm);
        p.seg_c = levels_[L - 1].C * 2;
        p.nseg = T;
        for (int t = 0; t < T; ++t) p.a[t] = mid_x_ + slots[t] * mplane;
        p.out = bneck_x_;
        p.out_c = p.seg_c;
        DN_TRY(gemm(bneck_, kProNone, kEpiStore, kARows, p, s));
        DN_TRY(run_stage(bneck_blocks_, bneck_x_, 1, hm, wm, s));
        for (int l = 0; l < L; ++l) {
            const int h = sh.Hp >> l, w = sh.Wp >> l, Cl = levels_[l].C;
            const size_t plane = static_cast<size_t>(h) * w * Cl;
            const __half* rf = enc_x_[l] + slots[ref] * plane;
            GemmParams q = rows_params(1, h, w);
            q.seg_c = Cl;
            q.nseg = T;
            int wi = 0;
            for (int t = 0; t < T; ++t) {
                const __half* f = enc_x_[l] + slots[t] * plane;
                if (info_.use_warp && t != ref) {
                    // offset head: DW 3x3 over [ref, f] -> PW -> ReLU -> PW -> (dx, dy)
                    ++launches_;
                    prof_begin("offset_dw", static_cast<double>(h) * w * 6 * Cl * 2, 36.0 * h * w * Cl, s);
                    DN_TRY(launch_dw_pair(rf, f, wptr<float>(oh_dw_[l]), oh_d_, h, w, Cl, s));
                    prof_end(s);
                    GemmParams o = rows_params(1, h, w);
                    o.seg_c = 2 * Cl;
                    o.a[0] = oh_d_;
                    o.out = oh_h_;
                    o.out_c = Cl;
                    o.relu = 1;
                    DN_TRY(gemm(oh_pw1_[l], kProNone, kEpiStore, kARows, o, s));
                    o = rows_params(1, h, w);
                    o.seg_c = Cl;
                    o.a[0] = oh_h_;
                    o.out = offset_buf_;
                    o.out_c = 8;
                    DN_TRY(gemm(oh_pw2_[l], kProNone, kEpiStore, kARows, o, s));
                    __half* wb = warp_buf_ + wi * plane;
                    ++wi;
                    ++launches_;
                    prof_begin("warp", static_cast<double>(h) * w * (2 * Cl + 16) * 2, 8.0 * h * w * Cl, s);
                    DN_TRY(launch_warp_pixel(f, offset_buf_, 8, wb, 1, h, w, Cl, static_cast<float>(w - 1) / w,
                                             static_cast<float>(h - 1) / h, s));
                    prof_end(s);
                    f = wb;
                }
                q.a[t] = f;
            }
            q.out = fused_skip_[l];
            q.out_c = Cl;
            DN_TRY(gemm(tmix_[l], kProNone, kEpiStore, kARows, q, s));
            DN_TRY(run_stage(tmix_blocks_[l], fused_skip_[l], 1, h, w, s));
        }
        return decode_from(bneck_x_, 1, fused_skip_, beauty, beauty_stride, y, s);
    }
    // Temporal model of the C++ engine (nafnet_temporal.cu:363-503): middle on
    // the reference frame's deep feature (a copy: the middle runs in place),
    // per-level fused skip temporal_mix(concat(ref, mean_t warp?(nbr_t))).
    for (int l = 0; l < L; ++l) {
        const int h = sh.Hp >> l, w = sh.Wp >> l, Cl = levels_[l].C;
        const size_t plane = static_cast<size_t>(h) * w * Cl;
        const __half* rf = enc_x_[l] + slots[ref] * plane;
        GemmParams p = rows_params(1, h, w);
        p.seg_c = Cl;
        p.a_img_stride = 0;
        p.nseg = T;
        p.a[0] = rf;
        int si = 1;
        for (int t = 0; t < T; ++t) {
            if (t == ref) continue;
            const __half* nb = enc_x_[l] + slots[t] * plane;
            if (info_.use_warp) {
                GemmParams q = rows_params(1, h, w);
                q.seg_c = Cl;
                q.a_img_stride = 0;
                q.nseg = 2;
                q.a[0] = rf;
                q.a[1] = nb;
                q.out = offset_buf_;
                q.out_c = 8;
                DN_TRY(gemm(offset_heads_[l], kProNone, kEpiStore, kARows, q, s));
                __half* wb = warp_buf_ + (si - 1) * plane;
                ++launches_;
                prof_begin("warp", static_cast<double>(h) * w * (2 * Cl + 16) * 2, 8.0 * h * w * Cl, s);
                DN_TRY(launch_warp_pixel(nb, offset_buf_, 8, wb, 1, h, w, Cl, 1.f, 1.f, s));
                prof_end(s);
                nb = wb;
            }
            p.a[si++] = nb;
        }
        p.out = fused_skip_[l];
        p.out_c = Cl;
        DN_TRY(gemm(tmix_[l], kProNone, kEpiStore, kARows, p, s));
    }
    cudaError_t e = cudaMemcpyAsync(bneck_x_, mid_x_ + slots[ref] * mplane, mplane * 2, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) return dn_cuda_fail(e, "temporal: reference deep feature copy");
    return decode_from(bneck_x_, 1, fused_skip_, beauty, beauty_stride, y, s);
}

int Engine::forward(const __half* x, int N, int T, int C, int H, int W, __half* y, cudaStream_t s) {
    if (!x || !y) return dn_fail(DN_ERR_INVALID_ARG, "forward: null pointer");
    const bool temporal = info_.kind != 0;
    if (temporal && T != info_.num_frames) return dn_fail(DN_ERR_INVALID_ARG, "forward: frame count mismatch");
    if (!temporal && T != 1) return dn_fail(DN_ERR_INVALID_ARG, "forward: spatial model takes 4-D input");
    DeviceGuard dg(device_);
    Shape sh;
    DN_TRY(make_shape(N, T, C, H, W, sh));
    launches_ = 0;
    if (!temporal) {
        DN_TRY(encode_into(x, N, C * H * W, 0, s));
        return decode_from(mid_x_, N, enc_x_, x, C * H * W, y, s);
    }
    // Every frame of a clip through the shared encoder as one batch of T
    // images (slots 0 .. T-1), then the temporal tail on those slots.
    std::vector<int> slots(T);
    for (int t = 0; t < T; ++t) slots[t] = t;
    const int ref = T / 2;
    for (int n = 0; n < N; ++n) {
        const __half* clip = x + static_cast<size_t>(n) * T * C * H * W;
        DN_TRY(encode_into(clip, T, C * H * W, 0, s));
        DN_TRY(temporal_tail(slots.data(), clip + static_cast<size_t>(ref) * C * H * W, C * H * W,
                             y + static_cast<size_t>(n) * 3 * H * W, s));
    }
    return DN_OK;
}

int Engine::encode_frame(const __half* frame, int C, int H, int W, int slot, cudaStream_t s) {
    if (!frame) return dn_fail(DN_ERR_INVALID_ARG, "encode_frame: null pointer");
    if (info_.kind == 0) return dn_fail(DN_ERR_INVALID_ARG, "encode_frame: spatial models have no frame cache");
    if (slot < 0 || slot >= info_.num_frames) return dn_fail(DN_ERR_INVALID_ARG, "encode_frame: slot outside [0, T)");
    DeviceGuard dg(device_);
    Shape sh;
    DN_TRY(make_shape(1, info_.num_frames, C, H, W, sh));
    launches_ = 0;
    return encode_into(frame, 1, C * H * W, slot, s);
}

int Engine::decode_window(const int* slots, const __half* beauty, int C, int H, int W, __half* y, cudaStream_t s) {
    if (!slots || !beauty || !y) return dn_fail(DN_ERR_INVALID_ARG, "decode_window: null pointer");
    if (info_.kind == 0) return dn_fail(DN_ERR_INVALID_ARG, "decode_window: spatial models have no frame cache");
    for (int t = 0; t < info_.num_frames; ++t)
        if (slots[t] < 0 || slots[t] >= info_.num_frames)
            return dn_fail(DN_ERR_INVALID_ARG, "decode_window: slot outside [0, T)");
    DeviceGuard dg(device_);
    Shape sh;
    DN_TRY(make_shape(1, info_.num_frames, C, H, W, sh));
    return temporal_tail(slots, beauty, C * H * W, y, s);
}

int Engine::check_device(cudaStream_t s) {
    DeviceGuard dg(device_);
    cudaError_t e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return dn_cuda_fail(e, "stream synchronize");
    if (!err_) return DN_OK;
    uint32_t word = 0;
    e = cudaMemcpy(&word, err_, 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return dn_cuda_fail(e, "read device error word");
    if (word != 0) {
        cudaMemset(err_, 0, 4);
        return dn_fail_str(DN_ERR_DEVICE, "kernel reported device error word " + std::to_string(word));
    }
    return DN_OK;
}

}  // namespace dnb
