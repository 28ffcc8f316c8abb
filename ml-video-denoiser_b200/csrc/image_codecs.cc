// Image file codecs of the denoiser CLI: PNG (8/16-bit gray, gray+alpha,
// RGB, RGBA, 8-bit palette; non-interlaced), OpenEXR (single-part scanline
// files with HALF / FLOAT / UINT channels, NO / RLE / ZIPS / ZIP
// compression), binary PPM (P5/P6, 8/16-bit) and PFM (PF/Pf). Pixels cross
// the C-ABI as FP16 NCHW planes (1, C, H, W).
//
// Semantics follow the reference's src/io/image_io.cc and exr_io.cc:
//   * 8-bit images load as 3 channels (gray replicated, alpha dropped) with
//     value / 255 (image_io.cc:26-42, 72-84); 16-bit PNG samples keep their
//     high byte first, as the 8-bit loader there does;
//   * 8-bit saves clamp round(v * 255 + 0.5) (image_io.cc:45-61);
//   * EXR loads R, G, B when present, else Y, else the first channel, as
//     FP16 (exr_io.cc:76-114); EXR saves 1 (Y) or 3 (B, G, R) HALF channels
//     (exr_io.cc:150-196), here with ZIP compression.
// JPEG (the reference's stb writer/reader) is not built: DN_ERR_UNSUPPORTED.
#include <cuda_fp16.h>
#include <zlib.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "denoiser_b200_io.h"
#include "status.h"

namespace {

struct Image {
    int C = 0, H = 0, W = 0;
    std::vector<float> px;  // NCHW planes
};

struct CodecError {
    int code;
    std::string msg;
};

[[noreturn]] void fail(int code, const std::string& msg) { throw CodecError{code, msg}; }

std::string lower_ext(const std::string& path) {
    const auto dot = path.find_last_of('.');
    if (dot == std::string::npos) return "";
    std::string e = path.substr(dot + 1);
    for (auto& ch : e) ch = static_cast<char>(std::tolower(static_cast<unsigned char>(ch)));
    return e;
}

std::vector<uint8_t> read_file(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f) fail(DN_ERR_IO, "cannot open '" + path + "'");
    const auto n = static_cast<size_t>(f.tellg());
    std::vector<uint8_t> buf(n);
    f.seekg(0);
    if (n) f.read(reinterpret_cast<char*>(buf.data()), static_cast<std::streamsize>(n));
    if (!f) fail(DN_ERR_IO, "cannot read '" + path + "'");
    return buf;
}

void write_file(const std::string& path, const std::vector<uint8_t>& buf) {
    std::ofstream f(path, std::ios::binary);
    if (!f) fail(DN_ERR_IO, "cannot write '" + path + "'");
    f.write(reinterpret_cast<const char*>(buf.data()), static_cast<std::streamsize>(buf.size()));
    if (!f) fail(DN_ERR_IO, "cannot write '" + path + "'");
}

uint32_t be32(const uint8_t* p) { return (uint32_t(p[0]) << 24) | (uint32_t(p[1]) << 16) | (uint32_t(p[2]) << 8) | p[3]; }
void put_be32(std::vector<uint8_t>& v, uint32_t x) {
    for (int s = 24; s >= 0; s -= 8) v.push_back(static_cast<uint8_t>(x >> s));
}

std::vector<uint8_t> inflate_all(const uint8_t* src, size_t n, size_t expect) {
    std::vector<uint8_t> out(expect);
    z_stream zs{};
    if (inflateInit(&zs) != Z_OK) fail(DN_ERR_FORMAT, "zlib init failed");
    zs.next_in = const_cast<Bytef*>(src);
    zs.avail_in = static_cast<uInt>(n);
    zs.next_out = out.data();
    zs.avail_out = static_cast<uInt>(expect);
    const int rc = inflate(&zs, Z_FINISH);
    const size_t got = zs.total_out;
    inflateEnd(&zs);
    if ((rc != Z_STREAM_END && rc != Z_OK && rc != Z_BUF_ERROR) || got != expect)
        fail(DN_ERR_FORMAT, "compressed data is corrupt or has the wrong size");
    return out;
}

std::vector<uint8_t> deflate_all(const uint8_t* src, size_t n) {
    uLongf cap = compressBound(static_cast<uLong>(n));
    std::vector<uint8_t> out(cap);
    if (compress2(out.data(), &cap, src, static_cast<uLong>(n), 6) != Z_OK) fail(DN_ERR_FORMAT, "zlib compress failed");
    out.resize(cap);
    return out;
}

// ---------------------------------------------------------------------------
// PNG
// ---------------------------------------------------------------------------

const uint8_t kPngSig[8] = {0x89, 'P', 'N', 'G', '\r', '\n', 0x1a, '\n'};

int paeth(int a, int b, int c) {
    const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
    if (pa <= pb && pa <= pc) return a;
    return pb <= pc ? b : c;
}

Image png_decode(const std::vector<uint8_t>& f) {
    if (f.size() < 8 || std::memcmp(f.data(), kPngSig, 8) != 0) fail(DN_ERR_FORMAT, "not a PNG file");
    uint32_t W = 0, H = 0;
    int depth = 0, ctype = -1, interlace = 0;
    std::vector<uint8_t> idat, plte;
    size_t p = 8;
    bool seen_end = false;
    while (p + 8 <= f.size() && !seen_end) {
        const uint32_t len = be32(&f[p]);
        if (p + 12 + static_cast<size_t>(len) > f.size()) fail(DN_ERR_FORMAT, "truncated PNG chunk");
        const std::string type(reinterpret_cast<const char*>(&f[p + 4]), 4);
        const uint8_t* d = &f[p + 8];
        if (type == "IHDR") {
            if (len < 13) fail(DN_ERR_FORMAT, "bad PNG header");
            W = be32(d);
            H = be32(d + 4);
            depth = d[8];
            ctype = d[9];
            interlace = d[12];
        } else if (type == "PLTE") {
            plte.assign(d, d + len);
        } else if (type == "IDAT") {
            idat.insert(idat.end(), d, d + len);
        } else if (type == "IEND") {
            seen_end = true;
        }
        p += 12 + len;
    }
    if (W == 0 || H == 0 || W > (1u << 16) || H > (1u << 16)) fail(DN_ERR_FORMAT, "bad PNG size");
    if (interlace != 0) fail(DN_ERR_UNSUPPORTED, "interlaced PNG is not supported");
    int spp;  // samples per pixel
    switch (ctype) {
        case 0: spp = 1; break;
        case 2: spp = 3; break;
        case 3: spp = 1; break;
        case 4: spp = 2; break;
        case 6: spp = 4; break;
        default: fail(DN_ERR_FORMAT, "bad PNG color type");
    }
    if (!((depth == 8) || (depth == 16 && ctype != 3)))
        fail(DN_ERR_UNSUPPORTED, "PNG bit depth " + std::to_string(depth) + " is not supported (8 or 16)");
    if (ctype == 3 && plte.size() < 3) fail(DN_ERR_FORMAT, "palette PNG without a palette");
    const int bpp = spp * depth / 8;
    const size_t stride = static_cast<size_t>(W) * bpp;
    std::vector<uint8_t> raw = inflate_all(idat.data(), idat.size(), (stride + 1) * H);
    std::vector<uint8_t> prev(stride, 0), cur(stride);
    Image im;
    im.C = 3;
    im.H = static_cast<int>(H);
    im.W = static_cast<int>(W);
    im.px.resize(static_cast<size_t>(3) * W * H);
    const size_t plane = static_cast<size_t>(W) * H;
    for (uint32_t y = 0; y < H; ++y) {
        const uint8_t* row = &raw[y * (stride + 1)];
        const int ft = row[0];
        for (size_t i = 0; i < stride; ++i) {
            const int x = row[1 + i];
            const int a = i >= static_cast<size_t>(bpp) ? cur[i - bpp] : 0;
            const int b = prev[i];
            const int c = i >= static_cast<size_t>(bpp) ? prev[i - bpp] : 0;
            int v;
            switch (ft) {
                case 0: v = x; break;
                case 1: v = x + a; break;
                case 2: v = x + b; break;
                case 3: v = x + ((a + b) >> 1); break;
                case 4: v = x + paeth(a, b, c); break;
                default: fail(DN_ERR_FORMAT, "bad PNG filter type");
            }
            cur[i] = static_cast<uint8_t>(v);
        }
        for (uint32_t xq = 0; xq < W; ++xq) {
            // 8-bit sample s of this pixel (16-bit: the high byte, as an 8-bit loader keeps)
            auto sample = [&](int s) -> int { return cur[static_cast<size_t>(xq) * bpp + s * (depth / 8)]; };
            int rgb[3];
            if (ctype == 3) {
                const int idx = sample(0);
                if (static_cast<size_t>(idx) * 3 + 2 >= plte.size()) fail(DN_ERR_FORMAT, "PNG palette index out of range");
                for (int k = 0; k < 3; ++k) rgb[k] = plte[idx * 3 + k];
            } else if (spp <= 2) {
                rgb[0] = rgb[1] = rgb[2] = sample(0);
            } else {
                for (int k = 0; k < 3; ++k) rgb[k] = sample(k);
            }
            for (int k = 0; k < 3; ++k) im.px[k * plane + static_cast<size_t>(y) * W + xq] = static_cast<float>(rgb[k]) / 255.f;
        }
        std::swap(prev, cur);
    }
    return im;
}

uint8_t to_u8(float f) { return static_cast<uint8_t>(std::clamp(static_cast<int>(f * 255.f + 0.5f), 0, 255)); }

std::vector<uint8_t> png_encode(const Image& im) {
    if (im.C != 1 && im.C != 3 && im.C != 4) fail(DN_ERR_UNSUPPORTED, "PNG: 1, 3 or 4 channels");
    const int ctype = im.C == 1 ? 0 : (im.C == 3 ? 2 : 6);
    const size_t stride = static_cast<size_t>(im.W) * im.C, plane = static_cast<size_t>(im.W) * im.H;
    std::vector<uint8_t> raw((stride + 1) * im.H);
    for (int y = 0; y < im.H; ++y) {
        uint8_t* row = &raw[y * (stride + 1)];
        row[0] = 0;  // filter: none
        for (int x = 0; x < im.W; ++x)
            for (int c = 0; c < im.C; ++c) row[1 + static_cast<size_t>(x) * im.C + c] = to_u8(im.px[c * plane + static_cast<size_t>(y) * im.W + x]);
    }
    const auto z = deflate_all(raw.data(), raw.size());
    std::vector<uint8_t> out(kPngSig, kPngSig + 8);
    auto chunk = [&](const char* type, const std::vector<uint8_t>& data) {
        put_be32(out, static_cast<uint32_t>(data.size()));
        const size_t start = out.size();
        out.insert(out.end(), type, type + 4);
        out.insert(out.end(), data.begin(), data.end());
        const uLong crc = crc32(0L, &out[start], static_cast<uInt>(data.size() + 4));
        put_be32(out, static_cast<uint32_t>(crc));
    };
    std::vector<uint8_t> ihdr;
    put_be32(ihdr, static_cast<uint32_t>(im.W));
    put_be32(ihdr, static_cast<uint32_t>(im.H));
    ihdr.insert(ihdr.end(), {8, static_cast<uint8_t>(ctype), 0, 0, 0});
    chunk("IHDR", ihdr);
    chunk("IDAT", z);
    chunk("IEND", {});
    return out;
}

// ---------------------------------------------------------------------------
// OpenEXR (single-part scanline)
// ---------------------------------------------------------------------------

struct ExrChannel {
    std::string name;
    int type;  // 0 UINT, 1 HALF, 2 FLOAT
};

int exr_type_size(int t) { return t == 1 ? 2 : 4; }

template <typename T>
T rd(const uint8_t* p) {
    T v;
    std::memcpy(&v, p, sizeof(T));
    return v;
}

float half_bits_to_float(uint16_t h) {
    __half_raw r;
    r.x = h;
    return __half2float(__half(r));
}

uint16_t float_to_half_bits(float f) {
    const __half h = __float2half(f);
    return static_cast<__half_raw>(h).x;
}

// EXR "ZIP": bytes were interleaved (even bytes first, then odd) and
// delta-coded before deflate.
std::vector<uint8_t> exr_unzip(const uint8_t* src, size_t n, size_t expect) {
    std::vector<uint8_t> t = inflate_all(src, n, expect);
    for (size_t i = 1; i < t.size(); ++i) t[i] = static_cast<uint8_t>(t[i - 1] + t[i] - 128);
    std::vector<uint8_t> out(expect);
    const size_t half = (expect + 1) / 2;
    for (size_t i = 0; i < expect; ++i) out[i] = (i & 1) ? t[half + i / 2] : t[i / 2];
    return out;
}

std::vector<uint8_t> exr_zip(const std::vector<uint8_t>& src) {
    const size_t n = src.size(), half = (n + 1) / 2;
    std::vector<uint8_t> t(n);
    for (size_t i = 0; i < n; ++i) (i & 1 ? t[half + i / 2] : t[i / 2]) = src[i];
    for (size_t i = n; i-- > 1;) t[i] = static_cast<uint8_t>(t[i] - t[i - 1] + 128);
    return deflate_all(t.data(), t.size());
}

std::vector<uint8_t> exr_unrle(const uint8_t* src, size_t n, size_t expect) {
    std::vector<uint8_t> t;
    t.reserve(expect);
    size_t p = 0;
    while (p < n) {
        const int8_t c = static_cast<int8_t>(src[p++]);
        if (c < 0) {
            const size_t cnt = static_cast<size_t>(-c);
            if (p + cnt > n) fail(DN_ERR_FORMAT, "EXR RLE data is corrupt");
            t.insert(t.end(), src + p, src + p + cnt);
            p += cnt;
        } else {
            if (p >= n) fail(DN_ERR_FORMAT, "EXR RLE data is corrupt");
            t.insert(t.end(), static_cast<size_t>(c) + 1, src[p++]);
        }
    }
    if (t.size() != expect) fail(DN_ERR_FORMAT, "EXR RLE data has the wrong size");
    for (size_t i = 1; i < t.size(); ++i) t[i] = static_cast<uint8_t>(t[i - 1] + t[i] - 128);
    std::vector<uint8_t> out(expect);
    const size_t half = (expect + 1) / 2;
    for (size_t i = 0; i < expect; ++i) out[i] = (i & 1) ? t[half + i / 2] : t[i / 2];
    return out;
}

Image exr_decode(const std::vector<uint8_t>& f) {
    if (f.size() < 8 || rd<uint32_t>(f.data()) != 20000630u) fail(DN_ERR_FORMAT, "not an OpenEXR file");
    const uint32_t ver = rd<uint32_t>(&f[4]);
    if (ver & 0x200) fail(DN_ERR_UNSUPPORTED, "tiled EXR is not supported");
    if (ver & 0x1800) fail(DN_ERR_UNSUPPORTED, "multi-part or deep EXR is not supported");
    size_t p = 8;
    std::vector<ExrChannel> chans;
    int comp = -1;
    int32_t xmin = 0, ymin = 0, xmax = -1, ymax = -1;
    auto cstr = [&](size_t& q) {
        const size_t s = q;
        while (q < f.size() && f[q]) ++q;
        if (q >= f.size()) fail(DN_ERR_FORMAT, "truncated EXR header");
        return std::string(reinterpret_cast<const char*>(&f[s]), q++ - s);
    };
    while (true) {
        if (p >= f.size()) fail(DN_ERR_FORMAT, "truncated EXR header");
        if (f[p] == 0) {
            ++p;
            break;
        }
        const std::string name = cstr(p), type = cstr(p);
        if (p + 4 > f.size()) fail(DN_ERR_FORMAT, "truncated EXR header");
        const int32_t size = rd<int32_t>(&f[p]);
        p += 4;
        if (size < 0 || p + static_cast<size_t>(size) > f.size()) fail(DN_ERR_FORMAT, "truncated EXR attribute");
        const uint8_t* v = &f[p];
        if (name == "channels" && type == "chlist") {
            size_t q = p;
            while (q < p + size && f[q]) {
                ExrChannel c;
                c.name = cstr(q);
                c.type = rd<int32_t>(&f[q]);
                const int32_t xs = rd<int32_t>(&f[q + 8]), ys = rd<int32_t>(&f[q + 12]);
                if (xs != 1 || ys != 1) fail(DN_ERR_UNSUPPORTED, "subsampled EXR channels are not supported");
                if (c.type < 0 || c.type > 2) fail(DN_ERR_FORMAT, "bad EXR pixel type");
                q += 16;
                chans.push_back(c);
            }
        } else if (name == "compression") {
            comp = v[0];
        } else if (name == "dataWindow") {
            xmin = rd<int32_t>(v);
            ymin = rd<int32_t>(v + 4);
            xmax = rd<int32_t>(v + 8);
            ymax = rd<int32_t>(v + 12);
        }
        p += size;
    }
    if (chans.empty()) fail(DN_ERR_FORMAT, "EXR without channels");
    const int64_t W = int64_t(xmax) - xmin + 1, H = int64_t(ymax) - ymin + 1;
    if (W <= 0 || H <= 0 || W > 65536 || H > 65536) fail(DN_ERR_FORMAT, "bad EXR data window");
    int lines;
    switch (comp) {
        case 0: case 1: case 2: lines = 1; break;  // NONE, RLE, ZIPS
        case 3: lines = 16; break;                  // ZIP
        default: fail(DN_ERR_UNSUPPORTED, "EXR compression " + std::to_string(comp) + " is not supported (NONE, RLE, ZIPS, ZIP)");
    }
    size_t line_bytes = 0;
    for (const auto& c : chans) line_bytes += static_cast<size_t>(W) * exr_type_size(c.type);
    const int64_t nchunks = (H + lines - 1) / lines;
    if (p + nchunks * 8 > f.size()) fail(DN_ERR_FORMAT, "truncated EXR offset table");
    // Output channels: R, G, B if present, else Y, else the first one.
    auto find = [&](const char* n) -> int {
        for (size_t i = 0; i < chans.size(); ++i)
            if (chans[i].name == n) return static_cast<int>(i);
        return -1;
    };
    std::vector<int> order;
    if (find("R") >= 0 && find("G") >= 0 && find("B") >= 0)
        order = {find("R"), find("G"), find("B")};
    else if (find("Y") >= 0)
        order = {find("Y")};
    else
        order = {0};
    Image im;
    im.C = static_cast<int>(order.size());
    im.H = static_cast<int>(H);
    im.W = static_cast<int>(W);
    im.px.assign(static_cast<size_t>(im.C) * W * H, 0.f);
    const size_t plane = static_cast<size_t>(W) * H;
    for (int64_t k = 0; k < nchunks; ++k) {
        const uint64_t off = rd<uint64_t>(&f[p + k * 8]);
        if (off + 8 > f.size()) fail(DN_ERR_FORMAT, "bad EXR chunk offset");
        const int32_t y0 = rd<int32_t>(&f[off]) - ymin;
        const int32_t sz = rd<int32_t>(&f[off + 4]);
        if (sz < 0 || off + 8 + static_cast<uint64_t>(sz) > f.size() || y0 < 0 || y0 >= H)
            fail(DN_ERR_FORMAT, "bad EXR chunk");
        const int nl = static_cast<int>(std::min<int64_t>(lines, H - y0));
        const size_t expect = line_bytes * nl;
        std::vector<uint8_t> buf;
        const uint8_t* data = &f[off + 8];
        if (static_cast<size_t>(sz) == expect) {
            buf.assign(data, data + expect);  // stored uncompressed (also allowed when compression does not pay)
        } else if (comp == 2 || comp == 3) {
            buf = exr_unzip(data, sz, expect);
        } else if (comp == 1) {
            buf = exr_unrle(data, sz, expect);
        } else {
            fail(DN_ERR_FORMAT, "EXR chunk has the wrong size");
        }
        size_t q = 0;
        for (int l = 0; l < nl; ++l) {
            const size_t row = static_cast<size_t>(y0 + l) * W;
            for (size_t ci = 0; ci < chans.size(); ++ci) {
                const int ts = exr_type_size(chans[ci].type);
                const int oc = static_cast<int>(std::find(order.begin(), order.end(), static_cast<int>(ci)) - order.begin());
                if (oc < im.C) {
                    float* dst = &im.px[oc * plane + row];
                    for (int64_t x = 0; x < W; ++x) {
                        const uint8_t* s = &buf[q + x * ts];
                        dst[x] = chans[ci].type == 1 ? half_bits_to_float(rd<uint16_t>(s))
                                 : chans[ci].type == 2 ? rd<float>(s)
                                                       : static_cast<float>(rd<uint32_t>(s));
                    }
                }
                q += static_cast<size_t>(W) * ts;
            }
        }
    }
    return im;
}

std::vector<uint8_t> exr_encode(const Image& im) {
    if (im.C != 1 && im.C != 3) fail(DN_ERR_UNSUPPORTED, "save_exr: only C=1 or C=3 supported, got C=" + std::to_string(im.C));
    // Channels in alphabetical order: B, G, R (planes 2, 1, 0) or Y.
    const std::vector<std::pair<std::string, int>> ch =
        im.C == 3 ? std::vector<std::pair<std::string, int>>{{"B", 2}, {"G", 1}, {"R", 0}}
                  : std::vector<std::pair<std::string, int>>{{"Y", 0}};
    std::vector<uint8_t> out;
    auto put = [&](const void* p, size_t n) { out.insert(out.end(), static_cast<const uint8_t*>(p), static_cast<const uint8_t*>(p) + n); };
    auto put_i32 = [&](int32_t v) { put(&v, 4); };
    auto attr = [&](const char* name, const char* type, const std::vector<uint8_t>& val) {
        put(name, std::strlen(name) + 1);
        put(type, std::strlen(type) + 1);
        put_i32(static_cast<int32_t>(val.size()));
        put(val.data(), val.size());
    };
    auto bytes_of = [](std::initializer_list<int32_t> v) {
        std::vector<uint8_t> b(v.size() * 4);
        std::memcpy(b.data(), v.begin(), b.size());
        return b;
    };
    const uint32_t magic = 20000630u, version = 2;
    put(&magic, 4);
    put(&version, 4);
    std::vector<uint8_t> chl;
    for (const auto& c : ch) {
        chl.insert(chl.end(), c.first.begin(), c.first.end());
        chl.push_back(0);
        const int32_t vals[4] = {1, 0, 1, 1};  // HALF, pLinear 0 + reserved, xSampling, ySampling
        const uint8_t* vb = reinterpret_cast<const uint8_t*>(vals);
        chl.insert(chl.end(), vb, vb + 16);
    }
    chl.push_back(0);
    attr("channels", "chlist", chl);
    attr("compression", "compression", {3});  // ZIP
    attr("dataWindow", "box2i", bytes_of({0, 0, im.W - 1, im.H - 1}));
    attr("displayWindow", "box2i", bytes_of({0, 0, im.W - 1, im.H - 1}));
    attr("lineOrder", "lineOrder", {0});
    {
        std::vector<uint8_t> v(4);
        const float one = 1.f;
        std::memcpy(v.data(), &one, 4);
        attr("pixelAspectRatio", "float", v);
        std::vector<uint8_t> c2(8, 0);
        attr("screenWindowCenter", "v2f", c2);
        attr("screenWindowWidth", "float", v);
    }
    out.push_back(0);  // end of header
    const int lines = 16;
    const int nchunks = (im.H + lines - 1) / lines;
    const size_t table = out.size();
    out.resize(out.size() + static_cast<size_t>(nchunks) * 8);
    const size_t plane = static_cast<size_t>(im.W) * im.H;
    for (int k = 0; k < nchunks; ++k) {
        const int y0 = k * lines, nl = std::min(lines, im.H - y0);
        std::vector<uint8_t> raw;
        raw.reserve(static_cast<size_t>(nl) * ch.size() * im.W * 2);
        for (int l = 0; l < nl; ++l)
            for (const auto& c : ch)
                for (int x = 0; x < im.W; ++x) {
                    const uint16_t hb = float_to_half_bits(im.px[c.second * plane + static_cast<size_t>(y0 + l) * im.W + x]);
                    raw.push_back(static_cast<uint8_t>(hb & 0xff));
                    raw.push_back(static_cast<uint8_t>(hb >> 8));
                }
        std::vector<uint8_t> z = exr_zip(raw);
        const std::vector<uint8_t>& data = z.size() < raw.size() ? z : raw;
        const uint64_t off = out.size();
        std::memcpy(&out[table + static_cast<size_t>(k) * 8], &off, 8);
        put_i32(y0);
        put_i32(static_cast<int32_t>(data.size()));
        put(data.data(), data.size());
    }
    return out;
}

// ---------------------------------------------------------------------------
// PPM (P5/P6) and PFM (Pf/PF)
// ---------------------------------------------------------------------------

Image pnm_decode(const std::vector<uint8_t>& f, bool pfm) {
    size_t p = 0;
    auto token = [&]() {
        while (p < f.size()) {
            if (std::isspace(f[p])) {
                ++p;
            } else if (f[p] == '#') {
                while (p < f.size() && f[p] != '\n') ++p;
            } else {
                break;
            }
        }
        const size_t s = p;
        while (p < f.size() && !std::isspace(f[p])) ++p;
        if (s == p) fail(DN_ERR_FORMAT, "truncated PNM/PFM header");
        return std::string(reinterpret_cast<const char*>(&f[s]), p - s);
    };
    const std::string magic = token();
    const int W = std::stoi(token()), H = std::stoi(token());
    const std::string third = token();
    ++p;  // one whitespace byte before the raster
    if (W <= 0 || H <= 0 || W > 65536 || H > 65536) fail(DN_ERR_FORMAT, "bad PNM/PFM size");
    Image im;
    im.H = H;
    im.W = W;
    const size_t plane = static_cast<size_t>(W) * H;
    if (pfm) {
        if (magic != "PF" && magic != "Pf") fail(DN_ERR_FORMAT, "not a PFM file");
        const int spp = magic == "PF" ? 3 : 1;
        const bool little = std::stof(third) < 0;
        if (!little) fail(DN_ERR_UNSUPPORTED, "big-endian PFM is not supported");
        if (p + plane * spp * 4 > f.size()) fail(DN_ERR_FORMAT, "truncated PFM raster");
        im.C = spp;
        im.px.resize(plane * spp);
        for (int y = 0; y < H; ++y)  // rows stored bottom to top
            for (int x = 0; x < W; ++x)
                for (int c = 0; c < spp; ++c)
                    im.px[c * plane + static_cast<size_t>(H - 1 - y) * W + x] = rd<float>(&f[p + ((static_cast<size_t>(y) * W + x) * spp + c) * 4]);
        return im;
    }
    if (magic != "P6" && magic != "P5") fail(DN_ERR_FORMAT, "not a binary PPM/PGM file");
    const int spp = magic == "P6" ? 3 : 1;
    const int maxv = std::stoi(third);
    if (maxv <= 0 || maxv > 65535) fail(DN_ERR_FORMAT, "bad PPM maxval");
    const int bps = maxv > 255 ? 2 : 1;
    if (p + plane * spp * bps > f.size()) fail(DN_ERR_FORMAT, "truncated PPM raster");
    im.C = 3;
    im.px.resize(plane * 3);
    for (size_t i = 0; i < plane; ++i)
        for (int c = 0; c < 3; ++c) {
            const size_t at = p + (i * spp + (spp == 3 ? c : 0)) * bps;
            const int v = bps == 2 ? (f[at] << 8 | f[at + 1]) : f[at];
            im.px[c * plane + i] = static_cast<float>(v) / static_cast<float>(maxv);
        }
    return im;
}

std::vector<uint8_t> pnm_encode(const Image& im, bool pfm) {
    const size_t plane = static_cast<size_t>(im.W) * im.H;
    std::string hdr;
    std::vector<uint8_t> out;
    if (pfm) {
        if (im.C != 1 && im.C != 3) fail(DN_ERR_UNSUPPORTED, "PFM: 1 or 3 channels");
        hdr = std::string(im.C == 3 ? "PF" : "Pf") + "\n" + std::to_string(im.W) + " " + std::to_string(im.H) + "\n-1.0\n";
        out.assign(hdr.begin(), hdr.end());
        for (int y = im.H - 1; y >= 0; --y)
            for (int x = 0; x < im.W; ++x)
                for (int c = 0; c < im.C; ++c) {
                    const float v = im.px[c * plane + static_cast<size_t>(y) * im.W + x];
                    const uint8_t* b = reinterpret_cast<const uint8_t*>(&v);
                    out.insert(out.end(), b, b + 4);
                }
        return out;
    }
    if (im.C != 1 && im.C != 3) fail(DN_ERR_UNSUPPORTED, "PPM: 1 or 3 channels");
    hdr = std::string(im.C == 3 ? "P6" : "P5") + "\n" + std::to_string(im.W) + " " + std::to_string(im.H) + "\n255\n";
    out.assign(hdr.begin(), hdr.end());
    for (size_t i = 0; i < plane; ++i)
        for (int c = 0; c < im.C; ++c) out.push_back(to_u8(im.px[c * plane + i]));
    return out;
}

// ---------------------------------------------------------------------------

Image decode_any(const std::string& path) {
    const std::string e = lower_ext(path);
    const auto f = read_file(path);
    if (e == "png") return png_decode(f);
    if (e == "exr") return exr_decode(f);
    if (e == "ppm" || e == "pgm") return pnm_decode(f, false);
    if (e == "pfm") return pnm_decode(f, true);
    if (e == "jpg" || e == "jpeg") fail(DN_ERR_UNSUPPORTED, "JPEG is not supported by this build (PNG, EXR, PPM, PFM)");
    fail(DN_ERR_UNSUPPORTED, "unknown image extension '" + e + "'");
}

template <typename F>
int guard(const char* name, F&& fn) {
    try {
        fn();
        return DN_OK;
    } catch (const CodecError& e) {
        return dnb::dn_fail_str(e.code, std::string(name) + ": " + e.msg);
    } catch (const std::exception& e) {
        return dnb::dn_fail_str(DN_ERR_FORMAT, std::string(name) + ": " + e.what());
    }
}

}  // namespace

extern "C" {

int dn_image_probe(const char* path, int* channels, int* height, int* width) {
    if (!path || !channels || !height || !width) return dnb::dn_fail(DN_ERR_INVALID_ARG, "dn_image_probe: null argument");
    return guard("dn_image_probe", [&] {
        const Image im = decode_any(path);
        *channels = im.C;
        *height = im.H;
        *width = im.W;
    });
}

int dn_image_read(const char* path, void* half_nchw, int channels, int height, int width) {
    if (!path || !half_nchw) return dnb::dn_fail(DN_ERR_INVALID_ARG, "dn_image_read: null argument");
    return guard("dn_image_read", [&] {
        const Image im = decode_any(path);
        if (im.C != channels || im.H != height || im.W != width)
            fail(DN_ERR_INVALID_ARG, "the file's size differs from the buffer's");
        auto* out = static_cast<uint16_t*>(half_nchw);
        for (size_t i = 0; i < im.px.size(); ++i) out[i] = float_to_half_bits(im.px[i]);
    });
}

int dn_image_write(const char* path, const void* half_nchw, int channels, int height, int width) {
    if (!path || !half_nchw) return dnb::dn_fail(DN_ERR_INVALID_ARG, "dn_image_write: null argument");
    if (channels <= 0 || height <= 0 || width <= 0) return dnb::dn_fail(DN_ERR_INVALID_ARG, "dn_image_write: empty image");
    return guard("dn_image_write", [&] {
        Image im;
        im.C = channels;
        im.H = height;
        im.W = width;
        const auto* in = static_cast<const uint16_t*>(half_nchw);
        im.px.resize(static_cast<size_t>(channels) * height * width);
        for (size_t i = 0; i < im.px.size(); ++i) im.px[i] = half_bits_to_float(in[i]);
        const std::string e = lower_ext(path);
        if (e == "png")
            write_file(path, png_encode(im));
        else if (e == "exr")
            write_file(path, exr_encode(im));
        else if (e == "ppm" || e == "pgm")
            write_file(path, pnm_encode(im, false));
        else if (e == "pfm")
            write_file(path, pnm_encode(im, true));
        else if (e == "jpg" || e == "jpeg")
            fail(DN_ERR_UNSUPPORTED, "JPEG is not supported by this build (PNG, EXR, PPM, PFM)");
        else
            fail(DN_ERR_UNSUPPORTED, "unknown image extension '" + e + "'");
    });
}

}  // extern "C"
