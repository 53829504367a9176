// DFlashKit host interface in C++ over libdflashcuda's C ABI.
//
// The reference host is Swift (random1st/dflash-swift, Sources/DFlashKit); this header
// mirrors the parts of its interface that sit on the verify hot path, with the same
// names, argument meaning and error behaviour, for hosts written in C++:
//   * SmallMQuantizedMatmul (SmallMQuantizedMatmul.swift:27-225): constants, isEligible,
//     tiles, apply;
//   * QuantizedLinear / SmallMQuantizedLinear (:234-293): a quantized linear layer whose
//     call runs on dflash_qmm, sharing (never copying) the wrapped layer's arrays;
//   * enableSmallMQuantizedMatmul(in:) (:304-317): swaps every eligible layer of a module
//     tree and returns the count;
//   * rollbackGatedDeltaRound / rollbackGatedDeltaTree (called at
//     DFlashSpeculativeGenerator.swift:455-460): rebuild each gated-delta layer's
//     MambaCache (conv window, recurrent state) from the round's capture;
//   * acceptedPrefix, the greedy accept of a chain round (DFlashSpeculativeGenerator.swift:555-571);
//   * SpeculativeTreePlan and the accepted-path walk (SpeculativeTreeTests.swift:25-78,
//     DFlashDraftTree.swift:122-141).
// Arrays are device memory (DeviceArray); outputs that the reference's MLX runtime would
// allocate are allocated here with cudaMalloc and owned by the returned DeviceArray.
// Failures throw DFlashError carrying the library status, where the reference calls
// fatalError; there is no CPU path.
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <optional>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "dflash_cuda.h"

namespace dflashkit {

enum class DType { bfloat16, float32, uint32, int32 };
enum class QuantizationMode { affine, mxfp4 };

size_t itemSize(DType t);

class DFlashError : public std::runtime_error {
public:
    DFlashError(int status, const std::string& message);
    int status;
};

// A device array: pointer, shape (row-major, contiguous) and element type.  `owner`
// keeps an allocation made by this library alive; views of caller memory leave it empty.
struct DeviceArray {
    void* data = nullptr;
    std::vector<int64_t> shape;
    DType dtype = DType::bfloat16;
    std::shared_ptr<void> owner;

    int64_t dim(int axis) const;  // negative axes count from the end
    int64_t size() const;
    size_t nbytes() const { return (size_t)size() * itemSize(dtype); }
    DeviceArray reshaped(std::vector<int64_t> newShape) const;
    static DeviceArray view(void* data, std::vector<int64_t> shape, DType dtype);
    static DeviceArray allocate(std::vector<int64_t> shape, DType dtype);  // cudaMalloc, owned
};

// ------------------------------------------------------------------ modules

class Module {
public:
    virtual ~Module() = default;
    // Named children, in insertion order (a layer is a Module with no children).
    std::vector<std::pair<std::string, std::shared_ptr<Module>>> children;
    std::shared_ptr<Module>& child(const std::string& name);
    void freeze() { frozen_ = true; }
    bool isFrozen() const { return frozen_; }

private:
    bool frozen_ = false;
};

class QuantizedLinear : public Module {
public:
    QuantizedLinear(DeviceArray weight, std::optional<DeviceArray> bias, DeviceArray scales,
                    std::optional<DeviceArray> biases, int groupSize, int bits,
                    QuantizationMode mode = QuantizationMode::affine);
    // (outputFeatures, inputFeatures)
    std::pair<int64_t, int64_t> shape() const;
    // The stock op (MLX quantizedMatmul) is not part of this library: throws
    // DFLASH_ERR_UNSUPPORTED.  SmallMQuantizedLinear overrides it.
    virtual DeviceArray callAsFunction(const DeviceArray& x, dflash_stream_t stream = nullptr);

    DeviceArray weight;
    std::optional<DeviceArray> bias;
    DeviceArray scales;
    std::optional<DeviceArray> biases;
    int groupSize;
    int bits;
    QuantizationMode mode;
};

struct SmallMQuantizedMatmul {
    // The kernel covers every row count 1..16 (the reference's starts at 6 because below
    // that MLX's GEMV wins, :29-32; this library has no stock op to defer to) and two
    // 8-row MMA n-tiles (:36-40).
    static constexpr int minimumRows = 1;
    static constexpr int maximumRows = 16;
    static constexpr int rowsPerTile = 8;

    // Static half of the eligibility test (:193-201): affine mode with biases, and a
    // bit width / group size / shape dflash_qmm covers (wider than the reference's gate:
    // groups 32, 64, 128 and any N, K with K % group == 0).
    static bool isEligible(const QuantizedLinear& layer);
    // MMA n-tiles for `rows` (:205-207).
    static int tiles(int rows);
    // x bf16 [rows, inputFeatures] . dequant(weight)^T -> bf16 [rows, outputFeatures]
    // (:210-224), written to `out` when given, else to a new array.
    static DeviceArray apply(const DeviceArray& x, const DeviceArray& weight, const DeviceArray& scales,
                             const DeviceArray& biases, int rows, int outputFeatures, int inputFeatures,
                             int bits, int groupSize = 64, DeviceArray* out = nullptr,
                             dflash_stream_t stream = nullptr);
};

class SmallMQuantizedLinear final : public QuantizedLinear {
public:
    // Wraps an existing layer, sharing its arrays, and stays frozen (:240-252).
    explicit SmallMQuantizedLinear(const QuantizedLinear& other);
    // Flattens leading dimensions to rows, runs the kernel in passes of at most 16 rows
    // (x rows are read in place: no zero-padding copy), reshapes back and adds the
    // optional bias (:254-292).  bf16 input only; an ineligible layer throws
    // DFLASH_ERR_UNSUPPORTED (there is no stock op to fall through to).
    DeviceArray callAsFunction(const DeviceArray& x, dflash_stream_t stream = nullptr) override;
    bool kernelEligible() const { return kernelEligible_; }

private:
    bool kernelEligible_;
};

// Swaps every eligible QuantizedLinear in the tree under `model` (not `model` itself)
// for a SmallMQuantizedLinear; returns how many were swapped.  Idempotent: wrapped
// layers are never wrapped again, so a second call returns 0 (:304-317).
int enableSmallMQuantizedMatmul(Module& model);

// ------------------------------------------------------------------ gated-delta rollback

// One gated-delta layer's cache (MambaCache, Tests/DFlashKitTests/GatedDeltaRollbackTests.swift:90-99):
// slot 0 the conv window bf16 [kc-1, C], slot 1 the recurrent state fp32 [H, dv, dk].
struct MambaCache {
    DeviceArray convWindow;
    DeviceArray state;
};

// What a verify round captured for one gated-delta layer (mtpGatedDeltaCapturesKey,
// DFlashSpeculativeGenerator.swift:453): the pre-round cache and the round's per-row
// recurrence inputs.
struct GatedDeltaCapture {
    DeviceArray convWindow;  // bf16 [kc-1, C], pre-round
    DeviceArray state;       // fp32 [H, dv, dk], pre-round
    DeviceArray convInputs;  // bf16 [width, C]: the rows' inputs to the conv
    DeviceArray k;           // bf16 [width, Hk, dk] (after conv, L2-normalised); Hk divides H, each
                             // key head shared by H / Hk value heads (Hk = H: one head count)
    DeviceArray v;           // bf16 [width, H, dv]
    DeviceArray alpha;       // fp32 [width, H]
    DeviceArray beta;        // fp32 [width, H]
};

// Leaves every cache as a committed forward over rows 0 .. keep-1 would have:
// state = replay of those rows from the captured state, conv window = last kc-1 rows of
// [captured window || their conv inputs].  One capture per cache, in layer order.
void rollbackGatedDeltaRound(std::vector<MambaCache>& caches, const std::vector<GatedDeltaCapture>& captures,
                             int width, int keep, dflash_stream_t stream = nullptr);
// The same over a tree round's accepted path (keepRows, anchor first).
void rollbackGatedDeltaTree(std::vector<MambaCache>& caches, const std::vector<GatedDeltaCapture>& captures,
                            int width, const std::vector<int32_t>& keepRows, dflash_stream_t stream = nullptr);

// ------------------------------------------------------------------ speculative trees

class SpeculativeTreePlan {
public:
    struct RowSource {
        int path;   // index into paths
        int depth;  // position of the row in that path
        bool operator==(const RowSource& o) const { return path == o.path && depth == o.depth; }
    };

    // parents[0] == -1 (the anchor); parents[r] in [0, r) for r > 0.  Throws
    // std::invalid_argument otherwise.
    explicit SpeculativeTreePlan(std::vector<int> parents);
    static SpeculativeTreePlan chain(int rows);

    int rows() const { return (int)parents.size(); }
    std::vector<int> ancestors(int row) const;  // anchor first, the row last
    // [rows, prefix + rows] row-major, 1 where a row may attend: the whole prefix, its
    // ancestors and itself.
    std::vector<uint8_t> attentionMask(int prefix) const;
    std::vector<int32_t> positions(int offset) const;  // offset + depth
    bool isRootPath(const std::vector<int>& rows) const;

    std::vector<int> parents;
    std::vector<std::vector<int>> children;
    std::vector<int> depths;
    std::vector<std::vector<int>> paths;  // one per leaf, leaves in row order
    int pathLength = 0;
    std::vector<RowSource> rowSources;
};

// The greedy accept of a chain round on host logits (DFlashSpeculativeGenerator
// .acceptedPrefix, DFlashSpeculativeGenerator.swift:555-571): the target's token per row
// is the argmax of its logits (the first index among equal maxima), and `accepted` is the
// length of the leading run of proposals equal to them; targetTokens[accepted] is the
// bonus token committed after them.  targetLogits: float [proposals + 1, vocabulary]
// row-major.  On the device the same test is dflash_accept over the LM head's argmax keys.
struct AcceptOutcome {
    std::vector<int32_t> targetTokens;
    std::vector<int32_t> proposals;
    int accepted = 0;
};
AcceptOutcome acceptedPrefix(const std::vector<float>& targetLogits, int vocabulary,
                             const std::vector<int32_t>& proposals);

// From the anchor, step into the first child (row order) whose drafted token the target
// named, until none does: (accepted rows, anchor first; the target's next token).
std::pair<std::vector<int>, int> acceptedPath(const std::vector<int>& tokens, const SpeculativeTreePlan& plan,
                                              const std::vector<int>& targetTokens);

}  // namespace dflashkit
