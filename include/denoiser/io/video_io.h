// denoiser::io video helpers — source-compatible with the reference's
// include/denoiser/io/video_io.h:9-37. Like the reference
// (src/io/video_io.cc), they run the ffprobe / ffmpeg command-line tools in a
// subprocess and throw std::runtime_error when a tool is missing or fails;
// frames travel as PNG files.
#pragma once

#include <algorithm>
#include <array>
#include <cstdio>
#include <cstdlib>
#include <filesystem>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

#include <unistd.h>

namespace denoiser::io {

struct VideoInfo {
    int width = 0;
    int height = 0;
    double fps = 25.0;
    int num_frames = 0;  // -1 if unknown
};

namespace detail {

inline std::string shell_quote(const std::string& s) {
    std::string q = "'";
    for (char ch : s) q += ch == '\'' ? std::string("'\\''") : std::string(1, ch);
    return q + "'";
}

// Runs `cmd`, returns its output; throws if it cannot start or exits non-zero.
inline std::string run_tool(const std::string& tool, const std::string& args) {
    if (std::system(("command -v " + tool + " >/dev/null 2>&1").c_str()) != 0)
        throw std::runtime_error("video_io: '" + tool + "' not found on PATH");
    FILE* p = popen((tool + " " + args + " 2>&1").c_str(), "r");
    if (!p) throw std::runtime_error("video_io: cannot start " + tool);
    std::string out;
    std::array<char, 4096> buf{};
    while (fgets(buf.data(), static_cast<int>(buf.size()), p)) out += buf.data();
    const int rc = pclose(p);
    if (rc != 0) throw std::runtime_error("video_io: " + tool + " failed (" + std::to_string(rc) + "): " + out);
    return out;
}

}  // namespace detail

inline VideoInfo probe_video(const std::string& path) {
    const std::string out = detail::run_tool(
        "ffprobe", "-v error -select_streams v:0 -show_entries stream=width,height,r_frame_rate,nb_frames "
                   "-of default=noprint_wrappers=1 " + detail::shell_quote(path));
    VideoInfo info;
    info.num_frames = -1;
    std::istringstream in(out);
    std::string line;
    while (std::getline(in, line)) {
        const auto eq = line.find('=');
        if (eq == std::string::npos) continue;
        const std::string k = line.substr(0, eq), v = line.substr(eq + 1);
        if (k == "width") info.width = std::stoi(v);
        else if (k == "height") info.height = std::stoi(v);
        else if (k == "nb_frames" && v != "N/A") info.num_frames = std::stoi(v);
        else if (k == "r_frame_rate") {
            const auto sl = v.find('/');
            const double num = std::stod(v.substr(0, sl)), den = sl == std::string::npos ? 1.0 : std::stod(v.substr(sl + 1));
            if (den > 0) info.fps = num / den;
        }
    }
    if (info.width <= 0 || info.height <= 0) throw std::runtime_error("probe_video: no video stream in '" + path + "'");
    return info;
}

inline std::vector<std::string> extract_frames(const std::string& video_path, const std::string& output_dir,
                                               double fps = 0.0, double start_sec = 0.0, double end_sec = 0.0) {
    namespace fs = std::filesystem;
    fs::create_directories(output_dir);
    std::ostringstream a;
    a << "-y";
    if (start_sec > 0.0) a << " -ss " << start_sec;
    a << " -i " << detail::shell_quote(video_path);
    if (end_sec > start_sec && end_sec > 0.0) a << " -t " << (end_sec - start_sec);
    if (fps > 0.0) a << " -vf fps=" << fps;
    a << " -pix_fmt rgb24 -loglevel error " << detail::shell_quote((fs::path(output_dir) / "frame_%06d.png").string());
    detail::run_tool("ffmpeg", a.str());
    std::vector<std::string> paths;
    for (const auto& e : fs::directory_iterator(output_dir))
        if (e.path().extension() == ".png") paths.push_back(e.path().string());
    std::sort(paths.begin(), paths.end());
    if (paths.empty()) throw std::runtime_error("extract_frames: no frames extracted from '" + video_path + "'");
    return paths;
}

inline void encode_frames(const std::vector<std::string>& frame_paths, const std::string& output_path,
                          double fps = 25.0) {
    namespace fs = std::filesystem;
    if (frame_paths.empty()) throw std::runtime_error("encode_frames: frame_paths is empty");
    // The frames, in order, as symlinks of one numbered pattern.
    const fs::path tmp = fs::temp_directory_path() / ("denoiser_encode_" + std::to_string(::getpid()));
    fs::create_directories(tmp);
    for (size_t i = 0; i < frame_paths.size(); ++i) {
        char name[32];
        std::snprintf(name, sizeof(name), "f_%08zu.png", i);
        fs::create_symlink(fs::absolute(frame_paths[i]), tmp / name);
    }
    std::ostringstream a;
    a << "-y -framerate " << fps << " -i " << detail::shell_quote((tmp / "f_%08d.png").string())
      << " -c:v libx264 -preset fast -crf 18 -pix_fmt yuv420p -loglevel error " << detail::shell_quote(output_path);
    try {
        detail::run_tool("ffmpeg", a.str());
    } catch (...) {
        fs::remove_all(tmp);
        throw;
    }
    fs::remove_all(tmp);
}

}  // namespace denoiser::io
