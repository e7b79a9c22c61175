// The reference's positional .weights format (parser.zig:446-591) for the C++ host: the
// counterpart of darknet_zig_b200/weights.py, for the parameters around the fused kernels
// (biases, BN scales and rolling statistics, the layer's weights as opaque floats).
//
// A file is a header -- i32 major = 0, i32 minor = 2, i32 revision = 0, u64 seen
// (parser.zig:576-579) -- then each layer's vectors in network order, f32, no names or sizes:
//   convolutional  biases[n]; if batch_normalize: scales, rolling_mean, rolling_variance [n];
//                  weights[nweights]                               (parser.zig:535-543)
//   connected      biases[n]; weights[n * inputs]; if batch_normalize: the three BN vectors
//                                                                  (parser.zig:545-553)
//   batchnorm      scales, rolling_mean, rolling_variance [n]      (parser.zig:555-559)
// Loading reads the same order (parser.zig:460-530): `seen` is a u64 when
// major * 10 + minor >= 2 and both are below 1000, else an i32; major or minor above 1000
// marks transposed (inputs x outputs) connected weights; `flipped` conv weights are stored
// (nweights / n) x n. dontload / dontsave skip a layer, dontloadscales skips the BN vectors
// of a conv or connected layer on load. Errors throw std::runtime_error (the reference's
// loader returns an error). Little-endian hosts only, like the reference's files.
#pragma once

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>
#include <vector>

namespace dnb::weights {

enum class Kind { Convolutional, Connected, Batchnorm };

struct Layer {
    Kind kind = Kind::Batchnorm;
    int n = 0;            // filters / outputs / channels
    bool batch_normalize = false;
    size_t nweights = 0;  // conv: n * c/groups * size * size; connected: n * inputs
    size_t inputs = 0;    // connected only
    bool dontload = false, dontsave = false, dontloadscales = false, flipped = false;
    std::vector<float> biases, scales, rolling_mean, rolling_variance, weights;

    // sizes every vector the layer's kind carries (zero-filled)
    void allocate() {
        if (kind == Kind::Connected && nweights == 0) nweights = (size_t)n * inputs;
        const bool bn = kind == Kind::Batchnorm || batch_normalize;
        if (kind != Kind::Batchnorm) {
            biases.assign(n, 0.0f);
            weights.assign(nweights, 0.0f);
        }
        if (bn) {
            scales.assign(n, 0.0f);
            rolling_mean.assign(n, 0.0f);
            rolling_variance.assign(n, 0.0f);
        }
    }
};

namespace detail {
struct File {
    FILE *f = nullptr;
    std::string path;
    File(const std::string &p, const char *mode) : f(fopen(p.c_str(), mode)), path(p) {
        if (!f) throw std::runtime_error("weights: cannot open " + p);
    }
    ~File() {
        if (f) fclose(f);
    }
    File(const File &) = delete;
    File &operator=(const File &) = delete;
    void write(const void *p, size_t bytes) {
        if (bytes && fwrite(p, 1, bytes, f) != bytes) throw std::runtime_error("weights: short write to " + path);
    }
    void read(void *p, size_t bytes) {
        if (bytes && fread(p, 1, bytes, f) != bytes)
            throw std::runtime_error("weights: " + path + " ends inside a layer's parameters");
    }
    void put(const std::vector<float> &v) { write(v.data(), v.size() * sizeof(float)); }
    void get(std::vector<float> &v) { read(v.data(), v.size() * sizeof(float)); }
};
// rows x cols (row-major) -> cols x rows, as parser.zig:451-458
inline void transpose(std::vector<float> &a, size_t rows, size_t cols) {
    std::vector<float> t(a.size());
    for (size_t x = 0; x < rows; ++x)
        for (size_t y = 0; y < cols; ++y) t[y * rows + x] = a[x * cols + y];
    a.swap(t);
}
}  // namespace detail

// saveWeights (parser.zig:561-590)
inline void save(const std::string &path, const std::vector<Layer> &layers, uint64_t seen) {
    detail::File f(path, "wb");
    const int32_t head[3] = {0, 2, 0};
    f.write(head, sizeof(head));
    f.write(&seen, sizeof(seen));
    for (const Layer &l : layers) {
        if (l.dontsave) continue;
        switch (l.kind) {
        case Kind::Convolutional:
            f.put(l.biases);
            if (l.batch_normalize) {
                f.put(l.scales);
                f.put(l.rolling_mean);
                f.put(l.rolling_variance);
            }
            f.put(l.weights);
            break;
        case Kind::Connected:
            f.put(l.biases);
            f.put(l.weights);
            if (l.batch_normalize) {
                f.put(l.scales);
                f.put(l.rolling_mean);
                f.put(l.rolling_variance);
            }
            break;
        case Kind::Batchnorm:
            f.put(l.scales);
            f.put(l.rolling_mean);
            f.put(l.rolling_variance);
            break;
        }
    }
}

// loadWeightsUpto (parser.zig:497-530): fills allocated layers in place, returns seen
inline uint64_t load(const std::string &path, std::vector<Layer> &layers, size_t start = 0,
                     size_t cutoff = SIZE_MAX) {
    detail::File f(path, "rb");
    int32_t head[3];
    f.read(head, sizeof(head));
    const int32_t major = head[0], minor = head[1];
    uint64_t seen = 0;
    if (major * 10 + minor >= 2 && major < 1000 && minor < 1000) {
        f.read(&seen, sizeof(seen));
    } else {
        int32_t s = 0;
        f.read(&s, sizeof(s));
        seen = s > 0 ? (uint64_t)s : 0;
    }
    const bool transpose = major > 1000 || minor > 1000;
    for (size_t i = start; i < layers.size() && i < cutoff; ++i) {
        Layer &l = layers[i];
        if (l.dontload) continue;
        const bool bn = l.batch_normalize && !l.dontloadscales;
        switch (l.kind) {
        case Kind::Convolutional:
            f.get(l.biases);
            if (bn) {
                f.get(l.scales);
                f.get(l.rolling_mean);
                f.get(l.rolling_variance);
            }
            f.get(l.weights);
            if (l.flipped) detail::transpose(l.weights, l.nweights / l.n, (size_t)l.n);
            break;
        case Kind::Connected:
            f.get(l.biases);
            f.get(l.weights);
            if (transpose) detail::transpose(l.weights, l.inputs, (size_t)l.n);
            if (bn) {
                f.get(l.scales);
                f.get(l.rolling_mean);
                f.get(l.rolling_variance);
            }
            break;
        case Kind::Batchnorm:
            f.get(l.scales);
            f.get(l.rolling_mean);
            f.get(l.rolling_variance);
            break;
        }
    }
    return seen;
}

}  // namespace dnb::weights
