// denoiser — command-line front end of the B200 engine, a drop-in for the
// reference's `denoiser` binary (cli/main.cc): the same flags
// (cli/main.cc:43-58), input kinds (an image, a directory of images, a video
// through ffmpeg, or a directory of frames in temporal mode), output naming
// (:133-136, 254-256, 329-331) and console messages, over the C++ API in
// include/denoiser/.
//
// Beyond the reference:
//   --gpus N   split a directory (spatial or temporal) into N contiguous
//              segments, one host thread and one engine per device
//              (devices --device .. --device+N-1); temporal segments load
//              the T/2 halo frames on each side, so outputs are identical
//              to a single-GPU run;
//   temporal mode encodes every frame once (the engine's frame cache,
//   dn_model_encode_frame / dn_model_decode_window) instead of building and
//   encoding a T-frame clip per output frame (cli/main.cc:155-187, 260-267).
// Image formats: PNG, EXR, PPM/PGM, PFM (include/denoiser_b200_io.h).
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <exception>
#include <filesystem>
#include <iostream>
#include <mutex>
#include <stdexcept>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

#include "denoiser/io/exr_io.h"
#include "denoiser/io/image_io.h"
#include "denoiser/io/video_io.h"
#include "denoiser/models/nafnet.h"
#include "denoiser/models/nafnet_temporal.h"
#include "denoiser/tensor.h"
#include "denoiser/weight_loader.h"

namespace fs = std::filesystem;
using namespace denoiser;

namespace {

struct Args {
    std::string model_path, input_path, output_path;
    std::string mode = "spatial";
    int device = 0;
    int num_frames = 3;
    int gpus = 1;
    bool prefetch = false;
};

void usage(const char* prog) {
    std::cerr << "Usage: " << prog << " --model <manifest.json> --input <path> [options]\n"
              << "\n"
              << "Required:\n"
              << "  --model  PATH   manifest.json from export.py\n"
              << "  --input  PATH   image (PNG/EXR/PPM/PFM), image directory, or video (MP4/MOV)\n"
              << "\n"
              << "Options:\n"
              << "  --output PATH   output path (default: <input>_denoised.<ext>)\n"
              << "  --mode   MODE   spatial | temporal  (default: spatial)\n"
              << "  --frames N      temporal window size (default: 3; the model's own window is used)\n"
              << "  --device N      first CUDA device index (default: 0)\n"
              << "  --gpus   N      devices to shard a directory over (default: 1)\n"
              << "  --prefetch      upload all weights before first inference\n"
              << "  --help\n";
}

Args parse(int argc, char** argv) {
    Args a;
    auto value = [&](int& i) -> std::string {
        if (++i >= argc) throw std::runtime_error("missing value for " + std::string(argv[i - 1]));
        return argv[i];
    };
    for (int i = 1; i < argc; ++i) {
        const std::string_view f = argv[i];
        if (f == "--help" || f == "-h") {
            usage(argv[0]);
            std::exit(0);
        } else if (f == "--model") {
            a.model_path = value(i);
        } else if (f == "--input") {
            a.input_path = value(i);
        } else if (f == "--output") {
            a.output_path = value(i);
        } else if (f == "--mode") {
            a.mode = value(i);
        } else if (f == "--frames") {
            a.num_frames = std::stoi(value(i));
        } else if (f == "--device") {
            a.device = std::stoi(value(i));
        } else if (f == "--gpus") {
            a.gpus = std::stoi(value(i));
        } else if (f == "--prefetch") {
            a.prefetch = true;
        } else {
            throw std::runtime_error("unknown flag: " + std::string(f));
        }
    }
    if (a.model_path.empty()) throw std::runtime_error("--model is required");
    if (a.input_path.empty()) throw std::runtime_error("--input is required");
    if (a.mode != "spatial" && a.mode != "temporal") throw std::runtime_error("--mode must be spatial or temporal");
    if (a.gpus < 1) throw std::runtime_error("--gpus must be >= 1");
    return a;
}

std::string lower(std::string s) {
    for (auto& c : s) c = static_cast<char>(std::tolower(static_cast<unsigned char>(c)));
    return s;
}

bool is_video(const fs::path& p) {
    const auto e = lower(p.extension().string());
    return e == ".mp4" || e == ".mov" || e == ".avi" || e == ".mkv";
}

bool is_image(const fs::path& p) {
    const auto e = lower(p.extension().string());
    return e == ".png" || e == ".exr" || e == ".ppm" || e == ".pgm" || e == ".pfm" || e == ".jpg" || e == ".jpeg";
}

bool is_exr(const fs::path& p) { return lower(p.extension().string()) == ".exr"; }

Tensor load_any(const fs::path& p, cudaStream_t s) { return is_exr(p) ? io::load_exr(p.string(), s) : io::load_image(p.string(), s); }

void save_any(const Tensor& t, const fs::path& p, cudaStream_t s) {
    if (is_exr(p))
        io::save_exr(t, p.string(), s);
    else
        io::save_image(t, p.string(), s);
}

fs::path default_output(const fs::path& in) { return in.parent_path() / (in.stem().string() + "_denoised" + in.extension().string()); }

fs::path default_dir(const fs::path& in) {
    const fs::path d = in.filename().empty() ? in.parent_path() : in;
    return d.parent_path() / (d.filename().string() + "_denoised");
}

std::vector<fs::path> list_images(const fs::path& dir) {
    std::vector<fs::path> v;
    for (const auto& e : fs::directory_iterator(dir))
        if (e.is_regular_file() && is_image(e.path())) v.push_back(e.path());
    std::sort(v.begin(), v.end());
    return v;
}

// Contiguous segment [s, e) of rank r of w over n items (earlier ranks take
// the remainder), the rule of the engine's frame sharding.
void segment(int n, int w, int r, int& s, int& e) {
    const int base = n / w, extra = n % w;
    s = r * base + std::min(r, extra);
    e = s + base + (r < extra ? 1 : 0);
}

std::mutex g_print;
void say(const std::string& line) {
    std::lock_guard<std::mutex> lk(g_print);
    std::cout << line << "\n" << std::flush;
}

std::string join(const std::vector<int>& v) {
    std::string s;
    for (size_t i = 0; i < v.size(); ++i) s += (i ? "," : "") + std::to_string(v[i]);
    return s;
}

// Spatial directory segment [s, e) on `device`.
void spatial_worker(const Args& a, int device, const std::vector<fs::path>& images, int s, int e, const fs::path& out_dir) {
    CUDA_CHECK(cudaSetDevice(device));
    cudaStream_t cs = nullptr, ts = nullptr;
    CUDA_CHECK(cudaStreamCreate(&cs));
    CUDA_CHECK(cudaStreamCreate(&ts));
    WeightStore store(a.model_path);
    if (a.prefetch) store.prefetch_all(ts);
    NAFNet model(store);
    for (int i = s; i < e; ++i) {
        Tensor in = load_any(images[i], ts);
        CUDA_CHECK(cudaStreamSynchronize(ts));
        Tensor out = model.forward(in, cs);
        CUDA_CHECK(cudaStreamSynchronize(cs));
        save_any(out, out_dir / images[i].filename(), cs);
        say("  " + images[i].filename().string());
    }
    CUDA_CHECK(cudaStreamDestroy(cs));
    CUDA_CHECK(cudaStreamDestroy(ts));
}

// Temporal directory segment [s, e) on `device`: every frame of the segment
// and its halo is encoded once into slot f % T; each output decodes the
// window of clamped indices (cli/main.cc:171-173).
void temporal_worker(const Args& a, int device, const std::vector<fs::path>& images, int s, int e, const fs::path& out_dir) {
    CUDA_CHECK(cudaSetDevice(device));
    cudaStream_t cs = nullptr;
    CUDA_CHECK(cudaStreamCreate(&cs));
    int dev = device;
    dn_model* m = nullptr;
    detail::check(dn_model_create(a.model_path.c_str(), dev, &m));
    dn_model_info info{};
    detail::check(dn_model_get_info(m, &info));
    const int T = info.num_frames, r = T / 2, n = static_cast<int>(images.size());
    std::vector<int> held(T, -1);
    std::vector<Tensor> frames(T);
    for (int i = s; i < e; ++i) {
        std::vector<int> slots(T);
        for (int t = 0; t < T; ++t) {
            const int f = std::clamp(i + t - r, 0, n - 1);
            const int sl = f % T;
            if (held[sl] != f) {
                frames[sl] = load_any(images[f], cs);
                const auto& sh = frames[sl].shape();
                detail::check(dn_model_encode_frame(m, frames[sl].data(), static_cast<int>(sh[1]), static_cast<int>(sh[2]),
                                                    static_cast<int>(sh[3]), sl, cs));
                held[sl] = f;
            }
            slots[t] = sl;
        }
        const Tensor& beauty = frames[i % T];
        const auto& sh = beauty.shape();
        if (frames[slots[0]].shape() != sh || frames[slots[T - 1]].shape() != sh)
            throw std::runtime_error("Temporal inference requires all frames in a sequence to share shape");
        Tensor out = Tensor::empty({1, 3, sh[2], sh[3]}, DType::kFloat16, cs);
        detail::check(dn_model_decode_window(m, slots.data(), T, beauty.data(), static_cast<int>(sh[1]),
                                             static_cast<int>(sh[2]), static_cast<int>(sh[3]), out.data(), cs));
        detail::check(dn_model_sync(m, cs));
        save_any(out, out_dir / images[i].filename(), cs);
        say("  " + images[i].filename().string());
    }
    frames.clear();
    CUDA_CHECK(cudaStreamSynchronize(cs));
    dn_model_destroy(m);
    CUDA_CHECK(cudaStreamDestroy(cs));
}

// Runs fn(rank, device, s, e) on `gpus` threads; rethrows the first failure.
template <typename Fn>
void shard(int n, int gpus, int device0, Fn&& fn) {
    std::vector<std::thread> pool;
    std::vector<std::exception_ptr> errs(gpus);
    for (int r = 0; r < gpus; ++r) {
        int s = 0, e = 0;
        segment(n, gpus, r, s, e);
        if (s == e) continue;
        pool.emplace_back([&, r, s, e] {
            try {
                fn(device0 + r, s, e);
            } catch (...) {
                errs[r] = std::current_exception();
            }
        });
    }
    for (auto& t : pool) t.join();
    for (auto& ep : errs)
        if (ep) std::rethrow_exception(ep);
}

}  // namespace

int main(int argc, char** argv) {
    if (argc < 2) {
        usage(argv[0]);
        return 1;
    }
    Args a;
    try {
        a = parse(argc, argv);
    } catch (const std::exception& ex) {
        std::cerr << "Error: " << ex.what() << "\n";
        usage(argv[0]);
        return 1;
    }
    try {
        int count = 0;
        CUDA_CHECK(cudaGetDeviceCount(&count));
        if (a.device < 0 || a.device + a.gpus > count)
            throw std::runtime_error("CUDA device " + std::to_string(a.device + a.gpus - 1) + " not available (" +
                                     std::to_string(count) + " devices found)");
        CUDA_CHECK(cudaSetDevice(a.device));
        std::cout << "Loading model: " << a.model_path << "\n";
        WeightStore store(a.model_path);
        const fs::path in(a.input_path);
        const bool temporal = a.mode == "temporal" || store.manifest().architecture.type == "nafnet_temporal";

        if (temporal) {
            if (!fs::is_directory(in)) throw std::runtime_error("Temporal mode expects an input directory of frames");
            {
                NAFNetTemporal probe(store);
                std::cout << "Model: NAFNetTemporal, enc_channels=[" << join(probe.enc_channels())
                          << "], frames=" << probe.num_frames() << ", use_warp=" << (probe.use_warp() ? "true" : "false")
                          << "\n";
            }
            const auto images = list_images(in);
            if (images.empty()) throw std::runtime_error("Temporal mode found no input frames");
            const fs::path out_dir = a.output_path.empty() ? default_dir(in) : fs::path(a.output_path);
            fs::create_directories(out_dir);
            std::cout << "Processing " << images.size() << " frames temporally → " << out_dir.string() << "\n";
            shard(static_cast<int>(images.size()), a.gpus, a.device,
                  [&](int dev, int s, int e) { temporal_worker(a, dev, images, s, e, out_dir); });
            return 0;
        }

        {
            NAFNet probe(store);
            std::cout << "Model: NAFNet, enc_channels=[" << join(probe.enc_channels()) << "]\n";
        }
        if (is_video(in)) {
            const io::VideoInfo info = io::probe_video(in.string());
            std::cout << "Video: " << info.width << "×" << info.height << " @ " << info.fps << " fps\n";
            const fs::path tmp_in = fs::temp_directory_path() / "denoiser_in_frames";
            const fs::path tmp_out = fs::temp_directory_path() / "denoiser_out_frames";
            fs::create_directories(tmp_out);
            std::cout << "Extracting frames...\n";
            const auto paths = io::extract_frames(in.string(), tmp_in.string(), 0.0);
            std::vector<fs::path> frames(paths.begin(), paths.end());
            std::cout << "Denoising " << frames.size() << " frames...\n";
            shard(static_cast<int>(frames.size()), a.gpus, a.device,
                  [&](int dev, int s, int e) { spatial_worker(a, dev, frames, s, e, tmp_out); });
            std::vector<std::string> outs;
            for (const auto& f : frames) outs.push_back((tmp_out / f.filename()).string());
            const fs::path out = a.output_path.empty() ? default_output(in) : fs::path(a.output_path);
            std::cout << "Encoding → " << out.string() << "\n";
            io::encode_frames(outs, out.string(), info.fps);
            fs::remove_all(tmp_in);
            fs::remove_all(tmp_out);
        } else if (fs::is_directory(in)) {
            const fs::path out_dir = a.output_path.empty() ? default_dir(in) : fs::path(a.output_path);
            fs::create_directories(out_dir);
            const auto images = list_images(in);
            std::cout << "Processing " << images.size() << " images → " << out_dir.string() << "\n";
            shard(static_cast<int>(images.size()), a.gpus, a.device,
                  [&](int dev, int s, int e) { spatial_worker(a, dev, images, s, e, out_dir); });
        } else {
            cudaStream_t cs = nullptr;
            CUDA_CHECK(cudaStreamCreate(&cs));
            if (a.prefetch) store.prefetch_all(cs);
            NAFNet model(store);
            Tensor x = load_any(in, cs);
            Tensor y = model.forward(x, cs);
            CUDA_CHECK(cudaStreamSynchronize(cs));
            const fs::path out = a.output_path.empty() ? default_output(in) : fs::path(a.output_path);
            save_any(y, out, cs);
            std::cout << "Saved: " << out.string() << "\n";
            CUDA_CHECK(cudaStreamDestroy(cs));
        }
        return 0;
    } catch (const std::exception& ex) {
        std::cerr << "Fatal error: " << ex.what() << "\n";
        return 1;
    }
}
