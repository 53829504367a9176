// DFlashKit host interface in C++ (see dflashkit.hpp): every compute step is a call into
// libdflashcuda's C ABI; this file holds argument checks, shapes, allocation of the
// outputs the reference's runtime would allocate, and the host-side tree bookkeeping.
#include "dflashkit.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>

namespace dflashkit {

size_t itemSize(DType t) {
    switch (t) {
        case DType::bfloat16: return 2;
        case DType::float32:
        case DType::uint32:
        case DType::int32: return 4;
    }
    return 0;
}

DFlashError::DFlashError(int st, const std::string& message)
    : std::runtime_error("status " + std::to_string(st) + ": " + message), status(st) {}

namespace {

[[noreturn]] void raise(int status, const std::string& message) { throw DFlashError(status, message); }

void check(int status) {
    if (status != DFLASH_OK) raise(status, dflash_last_error());
}

void cudaCheck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) raise(DFLASH_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

std::string shapeString(const std::vector<int64_t>& s) {
    std::string out = "[";
    for (size_t i = 0; i < s.size(); ++i) out += (i ? ", " : "") + std::to_string(s[i]);
    return out + "]";
}

void expect(const DeviceArray& a, DType dtype, size_t rank, const char* what) {
    if (a.dtype != dtype || a.shape.size() != rank || (!a.data && a.size() > 0))
        raise(DFLASH_ERR_INVALID_ARGUMENT, std::string(what) + ": unexpected dtype, rank or null data " +
                                               shapeString(a.shape));
}

// The dflash_qmm workspace of (device, stream): grown on demand and kept for the
// process, like the per-stream scratch MLX keeps for its kernels.  Growing waits for the
// stream, so a kernel still reading the old buffer finishes first.
void* qmmWorkspace(size_t bytes, dflash_stream_t stream, size_t* have) {
    struct Slot {
        void* ptr = nullptr;
        size_t bytes = 0;
    };
    static std::mutex mu;
    static std::map<std::pair<int, void*>, Slot> slots;
    int dev = 0;
    cudaCheck(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    Slot& s = slots[{dev, reinterpret_cast<void*>(stream)}];
    if (s.bytes < bytes) {
        if (s.ptr) {
            cudaCheck(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)), "cudaStreamSynchronize");
            cudaCheck(cudaFree(s.ptr), "cudaFree");
            s.ptr = nullptr;
            s.bytes = 0;
        }
        cudaCheck(cudaMalloc(&s.ptr, bytes), "cudaMalloc(workspace)");
        s.bytes = bytes;
    }
    *have = s.bytes;
    return s.ptr;
}

}  // namespace

// ------------------------------------------------------------------ DeviceArray

int64_t DeviceArray::dim(int axis) const {
    const int n = (int)shape.size();
    const int a = axis < 0 ? axis + n : axis;
    if (a < 0 || a >= n) raise(DFLASH_ERR_INVALID_ARGUMENT, "axis " + std::to_string(axis) + " of " + shapeString(shape));
    return shape[a];
}

int64_t DeviceArray::size() const {
    int64_t n = 1;
    for (int64_t d : shape) n *= d;
    return n;
}

DeviceArray DeviceArray::reshaped(std::vector<int64_t> newShape) const {
    DeviceArray out = *this;
    out.shape = std::move(newShape);
    if (out.size() != size())
        raise(DFLASH_ERR_INVALID_ARGUMENT, "cannot reshape " + shapeString(shape) + " to " + shapeString(out.shape));
    return out;
}

DeviceArray DeviceArray::view(void* data, std::vector<int64_t> shape, DType dtype) {
    DeviceArray a;
    a.data = data;
    a.shape = std::move(shape);
    a.dtype = dtype;
    return a;
}

DeviceArray DeviceArray::allocate(std::vector<int64_t> shape, DType dtype) {
    DeviceArray a = view(nullptr, std::move(shape), dtype);
    if (a.nbytes() == 0) return a;
    void* p = nullptr;
    cudaCheck(cudaMalloc(&p, a.nbytes()), "cudaMalloc");
    a.data = p;
    a.owner = std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
    return a;
}

// ------------------------------------------------------------------ modules

std::shared_ptr<Module>& Module::child(const std::string& name) {
    for (auto& c : children)
        if (c.first == name) return c.second;
    children.emplace_back(name, nullptr);
    return children.back().second;
}

QuantizedLinear::QuantizedLinear(DeviceArray weight_, std::optional<DeviceArray> bias_, DeviceArray scales_,
                                 std::optional<DeviceArray> biases_, int groupSize_, int bits_,
                                 QuantizationMode mode_)
    : weight(std::move(weight_)), bias(std::move(bias_)), scales(std::move(scales_)), biases(std::move(biases_)),
      groupSize(groupSize_), bits(bits_), mode(mode_) {
    if (weight.dtype != DType::uint32 || weight.shape.size() != 2)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "QuantizedLinear: weight must be uint32 [N, K*bits/32]");
    if (bits < 1 || bits > 32 || groupSize < 1)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "QuantizedLinear: bad bits / group size");
}

std::pair<int64_t, int64_t> QuantizedLinear::shape() const {
    return {weight.dim(0), weight.dim(1) * 32 / bits};
}

DeviceArray QuantizedLinear::callAsFunction(const DeviceArray&, dflash_stream_t) {
    raise(DFLASH_ERR_UNSUPPORTED,
          "the stock MLX quantizedMatmul is not part of this library; wrap the layer in SmallMQuantizedLinear");
}

// ------------------------------------------------------------------ SmallMQuantizedMatmul

bool SmallMQuantizedMatmul::isEligible(const QuantizedLinear& layer) {
    if (layer.mode != QuantizationMode::affine || !layer.biases) return false;
    if (layer.scales.dtype != DType::bfloat16 || layer.biases->dtype != DType::bfloat16) return false;
    const auto [outputFeatures, inputFeatures] = layer.shape();
    if (outputFeatures < 1 || inputFeatures < 1 || outputFeatures > INT32_MAX || inputFeatures > INT32_MAX)
        return false;
    return dflash_qmm_supported((int)outputFeatures, (int)inputFeatures, layer.groupSize, layer.bits) != 0;
}

int SmallMQuantizedMatmul::tiles(int rows) { return rows <= rowsPerTile ? 1 : 2; }

DeviceArray SmallMQuantizedMatmul::apply(const DeviceArray& x, const DeviceArray& weight, const DeviceArray& scales,
                                         const DeviceArray& biases, int rows, int outputFeatures, int inputFeatures,
                                         int bits, int groupSize, DeviceArray* out, dflash_stream_t stream) {
    if (rows < minimumRows || rows > maximumRows)
        raise(DFLASH_ERR_UNSUPPORTED, "SmallMQuantizedMatmul.apply: rows " + std::to_string(rows) + " outside 1..16");
    expect(x, DType::bfloat16, 2, "x");
    expect(weight, DType::uint32, 2, "weight");
    expect(scales, DType::bfloat16, 2, "scales");
    expect(biases, DType::bfloat16, 2, "biases");
    if (x.dim(0) < rows || x.dim(1) != inputFeatures || weight.dim(0) != outputFeatures)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "SmallMQuantizedMatmul.apply: x " + shapeString(x.shape) + ", weight " +
                                               shapeString(weight.shape) + " for rows " + std::to_string(rows));
    const size_t need = dflash_qmm_workspace_bytes(rows, outputFeatures, inputFeatures, groupSize, bits);
    if (need == 0 || !dflash_qmm_supported(outputFeatures, inputFeatures, groupSize, bits))
        raise(DFLASH_ERR_UNSUPPORTED, "SmallMQuantizedMatmul.apply: no kernel for this shape / format");
    DeviceArray y;
    if (out) {
        expect(*out, DType::bfloat16, 2, "out");
        if (out->dim(0) != rows || out->dim(1) != outputFeatures)
            raise(DFLASH_ERR_INVALID_ARGUMENT, "SmallMQuantizedMatmul.apply: out " + shapeString(out->shape));
        y = *out;
    } else {
        y = DeviceArray::allocate({rows, outputFeatures}, DType::bfloat16);
    }
    size_t have = 0;
    void* ws = qmmWorkspace(need, stream, &have);
    check(dflash_qmm(static_cast<const dflash_bf16*>(x.data), static_cast<const uint32_t*>(weight.data),
                     static_cast<const dflash_bf16*>(scales.data), static_cast<const dflash_bf16*>(biases.data),
                     static_cast<dflash_bf16*>(y.data), rows, outputFeatures, inputFeatures, groupSize, bits, ws,
                     have, stream));
    return y;
}

// ------------------------------------------------------------------ SmallMQuantizedLinear

SmallMQuantizedLinear::SmallMQuantizedLinear(const QuantizedLinear& other)
    : QuantizedLinear(other.weight, other.bias, other.scales, other.biases, other.groupSize, other.bits, other.mode),
      kernelEligible_(SmallMQuantizedMatmul::isEligible(other)) {
    freeze();
}

DeviceArray SmallMQuantizedLinear::callAsFunction(const DeviceArray& x, dflash_stream_t stream) {
    if (!kernelEligible_)
        raise(DFLASH_ERR_UNSUPPORTED, "SmallMQuantizedLinear: layer shape / format not covered by dflash_qmm");
    if (x.dtype != DType::bfloat16)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "SmallMQuantizedLinear takes bfloat16 input");
    if (x.shape.empty()) raise(DFLASH_ERR_INVALID_ARGUMENT, "SmallMQuantizedLinear: x has no feature axis");
    const auto [N, K] = shape();
    if (x.dim(-1) != K)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "SmallMQuantizedLinear: x " + shapeString(x.shape) + " for " +
                                               std::to_string(K) + " input features");
    const int64_t rows = x.size() / K;
    std::vector<int64_t> outShape(x.shape.begin(), x.shape.end() - 1);
    outShape.push_back(N);
    DeviceArray y = DeviceArray::allocate({rows, N}, DType::bfloat16);
    for (int64_t r0 = 0; r0 < rows; r0 += SmallMQuantizedMatmul::maximumRows) {
        const int n = (int)std::min<int64_t>(SmallMQuantizedMatmul::maximumRows, rows - r0);
        DeviceArray xp = DeviceArray::view(static_cast<uint16_t*>(x.data) + r0 * K, {n, K}, DType::bfloat16);
        DeviceArray yp = DeviceArray::view(static_cast<uint16_t*>(y.data) + r0 * N, {n, N}, DType::bfloat16);
        SmallMQuantizedMatmul::apply(xp, weight, scales, *biases, n, (int)N, (int)K, bits, groupSize, &yp, stream);
    }
    if (bias && rows > 0) {
        expect(*bias, DType::bfloat16, 1, "bias");
        if (bias->dim(0) != N) raise(DFLASH_ERR_INVALID_ARGUMENT, "SmallMQuantizedLinear: bias length");
        check(dflash_bias_add(static_cast<dflash_bf16*>(y.data), static_cast<const dflash_bf16*>(bias->data),
                              (int)rows, (int)N, stream));
    }
    return y.reshaped(outShape);
}

int enableSmallMQuantizedMatmul(Module& model) {
    int count = 0;
    std::unordered_map<const Module*, std::shared_ptr<Module>> wrapped;  // a shared layer gets one wrapper
    std::vector<Module*> stack{&model};
    std::unordered_map<const Module*, bool> seen;
    while (!stack.empty()) {
        Module* m = stack.back();
        stack.pop_back();
        if (seen[m]) continue;
        seen[m] = true;
        for (auto& [name, c] : m->children) {
            if (!c) continue;
            auto* q = dynamic_cast<QuantizedLinear*>(c.get());
            if (q) {
                if (dynamic_cast<SmallMQuantizedLinear*>(q) || !SmallMQuantizedMatmul::isEligible(*q)) continue;
                auto it = wrapped.find(q);
                if (it == wrapped.end()) it = wrapped.emplace(q, std::make_shared<SmallMQuantizedLinear>(*q)).first;
                c = it->second;
                ++count;
            } else {
                stack.push_back(c.get());
            }
        }
    }
    return count;
}

// ------------------------------------------------------------------ gated-delta rollback

namespace {

void rollback(std::vector<MambaCache>& caches, const std::vector<GatedDeltaCapture>& captures, int width,
              const int32_t* rows, int keep, dflash_stream_t stream) {
    if (caches.size() != captures.size())
        raise(DFLASH_ERR_INVALID_ARGUMENT, "rollback: " + std::to_string(captures.size()) + " captures for " +
                                               std::to_string(caches.size()) + " caches");
    for (size_t i = 0; i < caches.size(); ++i) {
        const GatedDeltaCapture& c = captures[i];
        MambaCache& m = caches[i];
        expect(c.state, DType::float32, 3, "capture state");
        expect(m.state, DType::float32, 3, "cache state");
        expect(c.k, DType::bfloat16, 3, "capture k");
        expect(c.v, DType::bfloat16, 3, "capture v");
        expect(c.alpha, DType::float32, 2, "capture alpha");
        expect(c.beta, DType::float32, 2, "capture beta");
        expect(c.convWindow, DType::bfloat16, 2, "capture conv window");
        expect(m.convWindow, DType::bfloat16, 2, "cache conv window");
        expect(c.convInputs, DType::bfloat16, 2, "capture conv inputs");
        const int64_t H = c.state.dim(0), dv = c.state.dim(1), dk = c.state.dim(2);
        const int64_t Hk = c.k.dim(1);  // key heads: each shared by H / Hk value heads
        if (Hk < 1 || H % Hk != 0 || m.state.shape != c.state.shape || c.k.shape != std::vector<int64_t>{width, Hk, dk} ||
            c.v.shape != std::vector<int64_t>{width, H, dv} || c.alpha.shape != std::vector<int64_t>{width, H} ||
            c.beta.shape != c.alpha.shape || m.convWindow.shape != c.convWindow.shape ||
            c.convInputs.dim(0) != width || c.convInputs.dim(1) != c.convWindow.dim(1))
            raise(DFLASH_ERR_INVALID_ARGUMENT, "rollback: layer " + std::to_string(i) + " shapes disagree");
        check(dflash_gdn_replay_grouped(static_cast<const float*>(c.state.data), static_cast<float*>(m.state.data),
                                        static_cast<const dflash_bf16*>(c.k.data),
                                        static_cast<const dflash_bf16*>(c.v.data),
                                        static_cast<const float*>(c.alpha.data), static_cast<const float*>(c.beta.data),
                                        rows, keep, width, 1, (int)H, (int)Hk, (int)dk, (int)dv, stream));
        check(dflash_gdn_conv_rollback(static_cast<const dflash_bf16*>(c.convWindow.data),
                                       static_cast<dflash_bf16*>(m.convWindow.data),
                                       static_cast<const dflash_bf16*>(c.convInputs.data), rows, keep, width, 1,
                                       (int)c.convWindow.dim(0), (int)c.convWindow.dim(1), stream));
    }
}

}  // namespace

void rollbackGatedDeltaRound(std::vector<MambaCache>& caches, const std::vector<GatedDeltaCapture>& captures,
                             int width, int keep, dflash_stream_t stream) {
    if (keep < 1 || keep > width)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "rollbackGatedDeltaRound: keep " + std::to_string(keep) + " of width " +
                                               std::to_string(width));
    rollback(caches, captures, width, nullptr, keep, stream);
}

void rollbackGatedDeltaTree(std::vector<MambaCache>& caches, const std::vector<GatedDeltaCapture>& captures,
                            int width, const std::vector<int32_t>& keepRows, dflash_stream_t stream) {
    if (keepRows.empty() || (int)keepRows.size() > width)
        raise(DFLASH_ERR_INVALID_ARGUMENT, "rollbackGatedDeltaTree: 1..width rows needed");
    for (int32_t r : keepRows)
        if (r < 0 || r >= width) raise(DFLASH_ERR_INVALID_ARGUMENT, "rollbackGatedDeltaTree: row outside the round");
    rollback(caches, captures, width, keepRows.data(), (int)keepRows.size(), stream);
}

// ------------------------------------------------------------------ speculative trees

SpeculativeTreePlan::SpeculativeTreePlan(std::vector<int> parents_) : parents(std::move(parents_)) {
    const int n = (int)parents.size();
    if (n == 0 || parents[0] != -1) throw std::invalid_argument("row 0 is the anchor: parents[0] must be -1");
    for (int r = 1; r < n; ++r)
        if (parents[r] < 0 || parents[r] >= r)
            throw std::invalid_argument("row " + std::to_string(r) + ": parent " + std::to_string(parents[r]) +
                                        " must be an earlier row");
    children.assign(n, {});
    depths.assign(n, 0);
    for (int r = 1; r < n; ++r) {
        children[parents[r]].push_back(r);
        depths[r] = depths[parents[r]] + 1;
    }
    for (int r = 0; r < n; ++r)
        if (children[r].empty()) paths.push_back(ancestors(r));
    for (const auto& p : paths) pathLength = std::max(pathLength, (int)p.size());
    rowSources.resize(n);
    for (int r = 0; r < n; ++r) {
        for (int i = 0; i < (int)paths.size(); ++i) {
            auto it = std::find(paths[i].begin(), paths[i].end(), r);
            if (it != paths[i].end()) {
                rowSources[r] = {i, (int)(it - paths[i].begin())};
                break;
            }
        }
    }
}

SpeculativeTreePlan SpeculativeTreePlan::chain(int rows) {
    std::vector<int> p(rows);
    for (int r = 0; r < rows; ++r) p[r] = r - 1;
    return SpeculativeTreePlan(p);
}

std::vector<int> SpeculativeTreePlan::ancestors(int row) const {
    std::vector<int> out{row};
    while (parents[out.back()] >= 0) out.push_back(parents[out.back()]);
    std::reverse(out.begin(), out.end());
    return out;
}

std::vector<uint8_t> SpeculativeTreePlan::attentionMask(int prefix) const {
    const int n = rows(), cols = prefix + n;
    std::vector<uint8_t> mask((size_t)n * cols, 0);
    for (int r = 0; r < n; ++r) {
        for (int c = 0; c < prefix; ++c) mask[(size_t)r * cols + c] = 1;
        for (int a : ancestors(r)) mask[(size_t)r * cols + prefix + a] = 1;
    }
    return mask;
}

std::vector<int32_t> SpeculativeTreePlan::positions(int offset) const {
    std::vector<int32_t> out(rows());
    for (int r = 0; r < rows(); ++r) out[r] = offset + depths[r];
    return out;
}

bool SpeculativeTreePlan::isRootPath(const std::vector<int>& rs) const {
    if (rs.empty() || rs[0] != 0) return false;
    for (size_t i = 1; i < rs.size(); ++i)
        if (rs[i] < 0 || rs[i] >= rows() || parents[rs[i]] != rs[i - 1]) return false;
    return true;
}

AcceptOutcome acceptedPrefix(const std::vector<float>& targetLogits, int vocabulary,
                             const std::vector<int32_t>& proposals) {
    const size_t rows = proposals.size() + 1;
    if (vocabulary < 1 || targetLogits.size() != rows * (size_t)vocabulary)
        throw std::invalid_argument("acceptedPrefix: logits must be [proposals + 1, vocabulary]");
    AcceptOutcome out;
    out.proposals = proposals;
    for (size_t r = 0; r < rows; ++r) {
        const float* row = targetLogits.data() + r * vocabulary;
        out.targetTokens.push_back((int32_t)(std::max_element(row, row + vocabulary) - row));  // first maximum
    }
    while (out.accepted < (int)proposals.size() && proposals[out.accepted] == out.targetTokens[out.accepted])
        ++out.accepted;
    return out;
}

std::pair<std::vector<int>, int> acceptedPath(const std::vector<int>& tokens, const SpeculativeTreePlan& plan,
                                              const std::vector<int>& targetTokens) {
    if ((int)tokens.size() != plan.rows() || (int)targetTokens.size() != plan.rows())
        throw std::invalid_argument("acceptedPath: one token and one target token per row");
    std::vector<int> rows{0};
    int row = 0;
    while (true) {
        int next = -1;
        for (int c : plan.children[row])
            if (tokens[c] == targetTokens[row]) {
                next = c;
                break;
            }
        if (next < 0) return {rows, targetTokens[row]};
        rows.push_back(next);
        row = next;
    }
}

}  // namespace dflashkit
