// Tests of the C++ host interface (dflash-swift_b200/host/dflashkit.hpp), laid out like
// the reference's XCTest cases they mirror:
//   cpu: SpeculativeTreeTests.swift:25-78 (plan shape), the accepted-path walk
//        (DFlashDraftTree.swift:122-141), AcceptLengthTests.swift:17-63 (the greedy
//        accept on one-peak logits), SmallMQuantizedMatmul eligibility and tiles
//        (SmallMQuantizedMatmul.swift:193-207), enableSmallMQuantizedMatmul's swap
//        semantics (:304-317) and the argument errors every entry reports before any
//        CUDA call;
//   gpu: SmallMQuantizedLinear against the qmm oracle (SmallMQuantizedMatmulTests.swift's
//        closeness measure, <= 1e-2), with bias and with more than 16 rows, and
//        rollbackGatedDeltaRound / Tree against the recurrence oracle
//        (GatedDeltaRollbackTests.swift:84-111: relative state error <= 1e-4, conv window
//        bit-exact);
//   stack <dir>: one verify round of the C-ABI stack object (include/dflash_stack.h) the
//        way a host drives it (DFlashSpeculativeGenerator.swift:389-398, :455-460,
//        :555-571): create over a shard's buffers, verify a block, commit the accepted
//        rows, advance.  The buffers come from <dir>/blob.bin as <dir>/manifest.txt
//        places them; what the round produced goes to <dir>/result.bin, placed by
//        <dir>/result.txt, for the test that wrote the inputs to compare.
// The oracle (oracle/liboracle.so) is the test's checker only.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <random>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "dflash_stack.h"
#include "dflashkit.hpp"

extern "C" {
uint16_t oracle_f32_to_bf16(float f);
float oracle_bf16_to_f32(uint16_t h);
void oracle_quantize_affine(const float* wf, int N, int K, int group, int bits, int refine, uint32_t* wq,
                            uint16_t* scales, uint16_t* biases);
void oracle_qmm_f64(const uint16_t* x, const uint32_t* w, const uint16_t* scales, const uint16_t* biases, int M,
                    int N, int K, int group, int bits, int flavour, double* y);
void oracle_gdn_recurrence(const float* s0, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                           const float* alpha, const float* beta, const int32_t* rows, int n_rows, int H, int dk,
                           int dv, double q_scale, double* s_out, double* o);
void oracle_conv_window(const uint16_t* window, const uint16_t* conv_in, const int32_t* rows, int n_rows, int kc1,
                        int C, uint16_t* out);
}

using namespace dflashkit;

static int g_failures = 0;
static int g_checks = 0;

#define CHECK(cond)                                                             \
    do {                                                                        \
        ++g_checks;                                                             \
        if (!(cond)) {                                                          \
            ++g_failures;                                                       \
            std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
        }                                                                       \
    } while (0)

// The status a call throws (DFlashError), 0 when it returns, -1 for another exception.
static int statusOf(const std::function<void()>& f) {
    try {
        f();
    } catch (const DFlashError& e) {
        return e.status;
    } catch (...) {
        return -1;
    }
    return 0;
}

static void* const kFake = reinterpret_cast<void*>(0x10000);  // never dereferenced by the cpu cases

static QuantizedLinear layer(int N, int K, int group, int bits, bool biases = true,
                             QuantizationMode mode = QuantizationMode::affine) {
    auto w = DeviceArray::view(kFake, {N, (int64_t)K * bits / 32}, DType::uint32);
    auto s = DeviceArray::view(kFake, {N, K / group}, DType::bfloat16);
    std::optional<DeviceArray> b;
    if (biases) b = s;
    return QuantizedLinear(w, std::nullopt, s, b, group, bits, mode);
}

// ------------------------------------------------------------------ cpu

static void testDepthsFollowTheTreeAndNotRowOrder() {
    SpeculativeTreePlan plan({-1, 0, 0, 1, 1, 3});
    CHECK((plan.depths == std::vector<int>{0, 1, 1, 2, 2, 3}));
}

static void testEveryLeafBecomesOneRootPath() {
    SpeculativeTreePlan plan({-1, 0, 0, 1, 1, 3});
    std::set<std::vector<int>> paths(plan.paths.begin(), plan.paths.end());
    CHECK((paths == std::set<std::vector<int>>{{0, 1, 3, 5}, {0, 1, 4}, {0, 2}}));
    CHECK(plan.pathLength == 4);
    for (int row = 0; row < plan.rows(); ++row) {
        const auto& src = plan.rowSources[row];
        CHECK(plan.paths[src.path][src.depth] == row);
    }
}

static void testAttentionMaskShowsAncestorsAndNothingElse() {
    SpeculativeTreePlan plan({-1, 0, 0, 1, 1, 3});
    const auto mask = plan.attentionMask(2);
    CHECK(mask.size() == 6u * 8u);
    auto sees = [&](int row, int col) { return mask[row * 8 + col] == 1; };
    for (int row = 0; row < 6; ++row) CHECK(sees(row, 0) && sees(row, 1));
    std::vector<int> five, two;
    for (int c = 0; c < 6; ++c) {
        if (sees(5, 2 + c)) five.push_back(c);
        if (sees(2, 2 + c)) two.push_back(c);
    }
    CHECK((five == std::vector<int>{0, 1, 3, 5}));
    CHECK((two == std::vector<int>{0, 2}));
}

static void testPositionsComeFromDepth() {
    SpeculativeTreePlan plan({-1, 0, 0, 1, 1, 3});
    CHECK((plan.positions(10) == std::vector<int32_t>{10, 11, 11, 12, 12, 13}));
}

static void testChainPlanIsTheDegenerateTree() {
    auto plan = SpeculativeTreePlan::chain(4);
    CHECK((plan.parents == std::vector<int>{-1, 0, 1, 2}));
    CHECK((plan.paths == std::vector<std::vector<int>>{{0, 1, 2, 3}}));
    CHECK(plan.isRootPath({0, 1, 2}));
    CHECK(!plan.isRootPath({0, 2}));
}

static void testMalformedParentsAreRejected() {
    auto throws = [](std::vector<int> p) {
        try {
            SpeculativeTreePlan plan(p);
        } catch (const std::invalid_argument&) {
            return true;
        }
        return false;
    };
    CHECK(throws({}));
    CHECK(throws({0, 0}));
    CHECK(throws({-1, 1}));
    CHECK(throws({-1, 0, 3}));
    CHECK(throws({-1, -1}));
}

static void testAcceptedPathWalksTheTargetsChoices() {
    SpeculativeTreePlan plan({-1, 0, 0, 1, 1, 3});
    const std::vector<int> tokens{11, 23, 37, 41, 37, 53};
    // target continues 11 -> 23 -> 37 (row 4, not row 2's 37: row 2 is not 1's child) -> 99
    auto [rows, bonus] = acceptedPath(tokens, plan, {23, 37, 0, 0, 99, 0});
    CHECK((rows == std::vector<int>{0, 1, 4}));
    CHECK(bonus == 99);
    auto [rows2, bonus2] = acceptedPath(tokens, plan, {37, 0, 5, 0, 0, 0});
    CHECK((rows2 == std::vector<int>{0, 2}));
    CHECK(bonus2 == 5);
    auto [rows3, bonus3] = acceptedPath(tokens, plan, {7, 0, 0, 0, 0, 0});
    CHECK((rows3 == std::vector<int>{0}));
    CHECK(bonus3 == 7);
    auto [rows4, bonus4] = acceptedPath(tokens, plan, {23, 41, 0, 53, 0, 8});
    CHECK((rows4 == std::vector<int>{0, 1, 3, 5}));
    CHECK(bonus4 == 8);
    CHECK(plan.isRootPath(rows4));
}

// AcceptLengthTests.swift:17-63: hand-built one-peak logits
static AcceptOutcome accept(const std::vector<int32_t>& target, const std::vector<int32_t>& proposals) {
    const int vocabulary = 10;
    std::vector<float> logits(target.size() * vocabulary, 0.f);
    for (size_t r = 0; r < target.size(); ++r) logits[r * vocabulary + target[r]] = 1.f;
    return acceptedPrefix(logits, vocabulary, proposals);
}

static void testAcceptLength() {
    auto full = accept({3, 4, 5, 6}, {3, 4, 5});
    CHECK(full.accepted == 3 && full.targetTokens[full.accepted] == 6);
    auto zero = accept({9, 4, 5, 6}, {3, 4, 5});
    CHECK(zero.accepted == 0 && zero.targetTokens[zero.accepted] == 9);
    auto partial = accept({3, 4, 8, 6, 1}, {3, 4, 5, 6});
    CHECK(partial.accepted == 2 && partial.targetTokens[partial.accepted] == 8);
    CHECK((partial.proposals == std::vector<int32_t>{3, 4, 5, 6}));
    std::vector<float> ties(2 * 5, 0.f);  // equal maxima resolve to the first index
    ties[1] = ties[3] = 2.f;
    ties[5 + 0] = ties[5 + 4] = 2.f;
    auto t = acceptedPrefix(ties, 5, {1});
    CHECK((t.targetTokens == std::vector<int32_t>{1, 0}) && t.accepted == 1);
    bool threw = false;
    try {
        acceptedPrefix(std::vector<float>(7), 5, {1});
    } catch (const std::invalid_argument&) {
        threw = true;
    }
    CHECK(threw);
}

static void testEligibilityAndTiles() {
    CHECK(SmallMQuantizedMatmul::isEligible(layer(4096, 1024, 64, 4)));
    CHECK(SmallMQuantizedMatmul::isEligible(layer(5120, 17408, 64, 8)));
    CHECK(SmallMQuantizedMatmul::isEligible(layer(1000, 640, 128, 4)));  // wider than the reference's gate
    CHECK(SmallMQuantizedMatmul::isEligible(layer(4096, 1024, 32, 4)));
    CHECK(!SmallMQuantizedMatmul::isEligible(layer(4096, 1024, 64, 4, /*biases=*/false)));
    CHECK(!SmallMQuantizedMatmul::isEligible(layer(4096, 1024, 64, 4, true, QuantizationMode::mxfp4)));
    CHECK(!SmallMQuantizedMatmul::isEligible(layer(4096, 1024, 64, 2)));
    CHECK(!SmallMQuantizedMatmul::isEligible(layer(4096, 1024, 16, 4)));
    CHECK(SmallMQuantizedMatmul::tiles(1) == 1 && SmallMQuantizedMatmul::tiles(8) == 1);
    CHECK(SmallMQuantizedMatmul::tiles(9) == 2 && SmallMQuantizedMatmul::tiles(16) == 2);
}

static void testArgumentErrorsComeBeforeAnyCudaCall() {
    auto w = DeviceArray::view(kFake, {4096, 128}, DType::uint32);
    auto s = DeviceArray::view(kFake, {4096, 16}, DType::bfloat16);
    auto x = DeviceArray::view(kFake, {8, 1024}, DType::bfloat16);
    auto apply = [&](const DeviceArray& xx, int rows, int group = 64) {
        return statusOf([&] { SmallMQuantizedMatmul::apply(xx, w, s, s, rows, 4096, 1024, 4, group); });
    };
    CHECK(apply(x, 17) == DFLASH_ERR_UNSUPPORTED);
    CHECK(apply(x, 0) == DFLASH_ERR_UNSUPPORTED);
    CHECK(apply(x, 9) == DFLASH_ERR_INVALID_ARGUMENT);                  // x holds 8 rows
    CHECK(apply(DeviceArray::view(kFake, {8, 1024}, DType::float32), 8) == DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(apply(DeviceArray::view(kFake, {8, 1000}, DType::bfloat16), 8) == DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(apply(x, 8, 48) == DFLASH_ERR_UNSUPPORTED);                   // no kernel for group 48

    SmallMQuantizedLinear inel(layer(4096, 1024, 64, 4, /*biases=*/false));
    CHECK(!inel.kernelEligible());
    CHECK(statusOf([&] { inel.callAsFunction(x); }) == DFLASH_ERR_UNSUPPORTED);
    SmallMQuantizedLinear ok(layer(4096, 1024, 64, 4));
    CHECK(ok.kernelEligible() && ok.isFrozen());
    CHECK(statusOf([&] { ok.callAsFunction(DeviceArray::view(kFake, {8, 1024}, DType::float32)); }) ==
          DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(statusOf([&] { ok.callAsFunction(DeviceArray::view(kFake, {8, 512}, DType::bfloat16)); }) ==
          DFLASH_ERR_INVALID_ARGUMENT);
    QuantizedLinear stock = layer(4096, 1024, 64, 4);
    CHECK(statusOf([&] { stock.callAsFunction(x); }) == DFLASH_ERR_UNSUPPORTED);

    std::vector<MambaCache> caches(2);
    std::vector<GatedDeltaCapture> captures(1);
    CHECK(statusOf([&] { rollbackGatedDeltaRound(caches, captures, 8, 4); }) == DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(statusOf([&] { rollbackGatedDeltaRound(caches, captures, 8, 0); }) == DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(statusOf([&] { rollbackGatedDeltaTree(caches, captures, 8, {0, 9}); }) == DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(statusOf([&] { rollbackGatedDeltaTree(caches, captures, 8, {}); }) == DFLASH_ERR_INVALID_ARGUMENT);
}

static void testEnableSwapsEligibleLayersOnceAndSharesArrays() {
    Module model;
    auto block = std::make_shared<Module>();
    auto attn = std::make_shared<Module>();
    auto q = std::make_shared<QuantizedLinear>(layer(4096, 1024, 64, 4));
    auto shared = std::make_shared<QuantizedLinear>(layer(5120, 2048, 64, 8));
    attn->child("q_proj") = q;
    attn->child("o_proj") = shared;
    attn->child("no_biases") = std::make_shared<QuantizedLinear>(layer(4096, 1024, 64, 4, false));
    block->child("attn") = attn;
    block->child("tied") = shared;  // the same layer at a second path
    model.child("layers.0") = block;
    model.child("norm") = std::make_shared<Module>();

    CHECK(enableSmallMQuantizedMatmul(model) == 3);
    auto* wrapped = dynamic_cast<SmallMQuantizedLinear*>(attn->child("q_proj").get());
    CHECK(wrapped != nullptr);
    CHECK(wrapped && wrapped->weight.data == q->weight.data && wrapped->scales.data == q->scales.data);
    CHECK(wrapped && wrapped->isFrozen());
    CHECK(dynamic_cast<SmallMQuantizedLinear*>(attn->child("no_biases").get()) == nullptr);
    CHECK(attn->child("o_proj").get() == block->child("tied").get());  // one wrapper for one layer
    CHECK(enableSmallMQuantizedMatmul(model) == 0);                   // idempotent
}

static int runCpu() {
    testDepthsFollowTheTreeAndNotRowOrder();
    testEveryLeafBecomesOneRootPath();
    testAttentionMaskShowsAncestorsAndNothingElse();
    testPositionsComeFromDepth();
    testChainPlanIsTheDegenerateTree();
    testMalformedParentsAreRejected();
    testAcceptedPathWalksTheTargetsChoices();
    testAcceptLength();
    testEligibilityAndTiles();
    testArgumentErrorsComeBeforeAnyCudaCall();
    testEnableSwapsEligibleLayersOnceAndSharesArrays();
    return 0;
}

// ------------------------------------------------------------------ gpu

template <class T>
static DeviceArray upload(const std::vector<T>& h, std::vector<int64_t> shape, DType dtype) {
    auto a = DeviceArray::allocate(std::move(shape), dtype);
    if (cudaMemcpy(a.data, h.data(), a.nbytes(), cudaMemcpyHostToDevice) != cudaSuccess) throw std::runtime_error("H2D");
    return a;
}

template <class T>
static std::vector<T> download(const DeviceArray& a) {
    std::vector<T> h(a.nbytes() / sizeof(T));
    if (cudaMemcpy(h.data(), a.data, a.nbytes(), cudaMemcpyDeviceToHost) != cudaSuccess) throw std::runtime_error("D2H");
    return h;
}

static std::vector<uint16_t> randomBf16(size_t n, std::mt19937& rng, float scale = 1.f) {
    std::normal_distribution<float> d(0.f, scale);
    std::vector<uint16_t> out(n);
    for (auto& v : out) v = oracle_f32_to_bf16(d(rng));
    return out;
}

static double closeness(const std::vector<double>& got, const std::vector<double>& want) {
    double diff = 0, scale = 1;
    for (size_t i = 0; i < got.size(); ++i) {
        diff = std::max(diff, std::fabs(got[i] - want[i]));
        scale = std::max(scale, std::fabs(want[i]));
    }
    return diff / scale;
}

static void testSmallMQuantizedLinearMatchesTheOracle(int rows, bool withBias) {
    const int N = 4096, K = 1024, group = 64, bits = 4;
    std::mt19937 rng(rows * 7 + withBias);
    std::normal_distribution<float> d(0.f, 0.02f);
    std::vector<float> wf((size_t)N * K);
    for (auto& v : wf) v = d(rng);
    std::vector<uint32_t> wq((size_t)N * K * bits / 32);
    std::vector<uint16_t> sc((size_t)N * K / group), bi((size_t)N * K / group);
    oracle_quantize_affine(wf.data(), N, K, group, bits, 1, wq.data(), sc.data(), bi.data());
    const auto x = randomBf16((size_t)rows * K, rng);
    const auto bias = randomBf16(N, rng, 0.5f);
    std::optional<DeviceArray> biasArr;
    if (withBias) biasArr = upload(bias, {N}, DType::bfloat16);
    QuantizedLinear base(upload(wq, {N, K * bits / 32}, DType::uint32), biasArr,
                         upload(sc, {N, K / group}, DType::bfloat16), upload(bi, {N, K / group}, DType::bfloat16),
                         group, bits);
    Module model;
    model.child("proj") = std::make_shared<QuantizedLinear>(base);
    CHECK(enableSmallMQuantizedMatmul(model) == 1);
    auto& linear = dynamic_cast<SmallMQuantizedLinear&>(*model.child("proj"));
    // leading dimensions [rows / 2, 2] when rows is even: flattened and restored
    std::vector<int64_t> xs = rows % 2 ? std::vector<int64_t>{rows, K} : std::vector<int64_t>{rows / 2, 2, K};
    auto y = linear.callAsFunction(upload(x, xs, DType::bfloat16));
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    CHECK(y.shape.size() == xs.size() && y.dim(-1) == N && y.size() == (int64_t)rows * N);
    const auto yh = download<uint16_t>(y);
    std::vector<double> want((size_t)rows * N), got((size_t)rows * N);
    oracle_qmm_f64(x.data(), wq.data(), sc.data(), bi.data(), rows, N, K, group, bits, 0, want.data());
    for (size_t i = 0; i < want.size(); ++i) {
        if (withBias) want[i] += oracle_bf16_to_f32(bias[i % N]);
        got[i] = oracle_bf16_to_f32(yh[i]);
    }
    const double c = closeness(got, want);
    if (c > 1e-2) std::fprintf(stderr, "rows %d bias %d: closeness %g\n", rows, (int)withBias, c);
    CHECK(c <= 1e-2);
}

static void testRollbackMatchesTheOracle(bool tree, int Hk = 4) {
    const int L = 2, W = 8, H = 4, dk = 128, dv = 128, kc1 = 3, C = 384;
    std::mt19937 rng(tree ? 3 : 4);
    std::normal_distribution<float> n01(0.f, 1.f);
    std::uniform_real_distribution<float> ua(0.9f, 1.f), ub(0.f, 1.f);
    const std::vector<int32_t> rows = tree ? std::vector<int32_t>{0, 2, 5} : std::vector<int32_t>{0, 1, 2, 3, 4};
    const int keep = (int)rows.size();
    std::vector<GatedDeltaCapture> caps;
    std::vector<MambaCache> caches;
    struct Host {
        std::vector<float> s0, a, b;
        std::vector<uint16_t> k, v, win, cin;
    };
    std::vector<Host> hosts(L);
    for (int l = 0; l < L; ++l) {
        Host& h = hosts[l];
        h.s0.resize((size_t)H * dv * dk);
        for (auto& v : h.s0) v = 0.1f * n01(rng);
        std::vector<float> kf((size_t)W * Hk * dk);  // Hk key heads, each read by H / Hk value heads
        for (auto& v : kf) v = n01(rng);
        for (int t = 0; t < W * Hk; ++t) {  // L2-normalised per head
            double ss = 0;
            for (int j = 0; j < dk; ++j) ss += (double)kf[(size_t)t * dk + j] * kf[(size_t)t * dk + j];
            for (int j = 0; j < dk; ++j) kf[(size_t)t * dk + j] = (float)(kf[(size_t)t * dk + j] / std::sqrt(ss));
        }
        h.k.resize(kf.size());
        for (size_t i = 0; i < kf.size(); ++i) h.k[i] = oracle_f32_to_bf16(kf[i]);
        h.v = randomBf16((size_t)W * H * dv, rng);
        h.a.resize((size_t)W * H);
        h.b.resize((size_t)W * H);
        for (auto& v : h.a) v = ua(rng);
        for (auto& v : h.b) v = ub(rng);
        h.win = randomBf16((size_t)kc1 * C, rng);
        h.cin = randomBf16((size_t)W * C, rng);
        GatedDeltaCapture c;
        c.state = upload(h.s0, {H, dv, dk}, DType::float32);
        c.k = upload(h.k, {W, Hk, dk}, DType::bfloat16);
        c.v = upload(h.v, {W, H, dv}, DType::bfloat16);
        c.alpha = upload(h.a, {W, H}, DType::float32);
        c.beta = upload(h.b, {W, H}, DType::float32);
        c.convWindow = upload(h.win, {kc1, C}, DType::bfloat16);
        c.convInputs = upload(h.cin, {W, C}, DType::bfloat16);
        caps.push_back(c);
        caches.push_back({DeviceArray::allocate({kc1, C}, DType::bfloat16),
                          DeviceArray::allocate({H, dv, dk}, DType::float32)});
    }
    if (tree)
        rollbackGatedDeltaTree(caches, caps, W, rows);
    else
        rollbackGatedDeltaRound(caches, caps, W, keep);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    for (int l = 0; l < L; ++l) {
        const Host& h = hosts[l];
        std::vector<uint16_t> kv((size_t)W * H * dk);  // k per value head for the oracle
        for (int t = 0; t < W; ++t)
            for (int hv = 0; hv < H; ++hv)
                std::memcpy(&kv[((size_t)t * H + hv) * dk], &h.k[((size_t)t * Hk + hv / (H / Hk)) * dk], dk * 2);
        std::vector<double> want((size_t)H * dv * dk);
        oracle_gdn_recurrence(h.s0.data(), nullptr, kv.data(), h.v.data(), h.a.data(), h.b.data(),
                              tree ? rows.data() : nullptr, keep, H, dk, dv, 1.0, want.data(), nullptr);
        const auto got = download<float>(caches[l].state);
        double diff = 0, scale = 0;
        for (size_t i = 0; i < want.size(); ++i) {
            diff = std::max(diff, std::fabs((double)got[i] - want[i]));
            scale = std::max(scale, std::fabs(want[i]));
        }
        CHECK(diff / scale <= 1e-4);
        std::vector<uint16_t> wantWin((size_t)kc1 * C);
        oracle_conv_window(h.win.data(), h.cin.data(), tree ? rows.data() : nullptr, keep, kc1, C, wantWin.data());
        CHECK(download<uint16_t>(caches[l].convWindow) == wantWin);
    }
}

static int runGpu() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n < 1) {
        std::fprintf(stderr, "no CUDA device\n");
        return 2;
    }
    testSmallMQuantizedLinearMatchesTheOracle(6, false);
    testSmallMQuantizedLinearMatchesTheOracle(8, true);
    testSmallMQuantizedLinearMatchesTheOracle(20, true);  // passes of 16 + 4 rows
    testSmallMQuantizedLinearMatchesTheOracle(1, false);
    testRollbackMatchesTheOracle(false);
    testRollbackMatchesTheOracle(true);
    testRollbackMatchesTheOracle(true, 2);  // shared key heads
    testRollbackMatchesTheOracle(false, 1);
    uint32_t bits = 0;
    CHECK(dflash_device_error(&bits, nullptr) == DFLASH_OK && bits == 0);
    return 0;
}

// ------------------------------------------------------------------ stack object

struct StackInputs {
    std::map<std::string, std::pair<size_t, size_t>> tensors;  // name -> (offset, bytes) in blob.bin
    std::map<std::string, std::pair<int, int>> qshape;          // quantized projection -> (N, K)
    std::map<std::string, double> cfg;
    std::vector<int> attention;                                 // per layer: 0 gated delta, 1 attention
    uint8_t* base = nullptr;                                    // blob.bin on the device
};

static bool readStackInputs(const std::string& dir, StackInputs& in) {
    std::ifstream mf(dir + "/manifest.txt");
    if (!mf) return false;
    std::string line;
    while (std::getline(mf, line)) {
        std::istringstream ls(line);
        std::string kind, name;
        ls >> kind >> name;
        if (kind == "cfg") {
            double v;
            ls >> v;
            in.cfg[name] = v;
        } else if (kind == "tensor") {
            size_t off, bytes;
            ls >> off >> bytes;
            in.tensors[name] = {off, bytes};
        } else if (kind == "qweight") {
            int N, K;
            ls >> N >> K;
            in.qshape[name] = {N, K};
        } else if (kind == "layer") {
            int att;
            ls >> att;
            in.attention.push_back(att);
        }
    }
    std::ifstream bf(dir + "/blob.bin", std::ios::binary);
    if (!bf) return false;
    std::vector<char> blob((std::istreambuf_iterator<char>(bf)), std::istreambuf_iterator<char>());
    if (cudaMalloc(&in.base, blob.size()) != cudaSuccess) return false;
    return cudaMemcpy(in.base, blob.data(), blob.size(), cudaMemcpyHostToDevice) == cudaSuccess;
}

static int runStack(const std::string& dir) {
    StackInputs in;
    if (!readStackInputs(dir, in)) {
        std::fprintf(stderr, "cannot read the stack inputs in %s\n", dir.c_str());
        return 2;
    }
    auto ptr = [&](const std::string& name) -> void* {
        auto it = in.tensors.find(name);
        return it == in.tensors.end() ? nullptr : in.base + it->second.first;
    };
    auto bf = [&](const std::string& name) { return static_cast<dflash_bf16*>(ptr(name)); };
    auto qw = [&](const std::string& name) {
        dflash_qweight q{};
        auto it = in.qshape.find(name);
        if (it == in.qshape.end()) return q;
        q.w = static_cast<const uint32_t*>(ptr(name + ".w"));
        q.scales = bf(name + ".scales");
        q.biases = bf(name + ".biases");
        q.N = it->second.first;
        q.K = it->second.second;
        return q;
    };
    auto cfg = [&](const char* key) { return (int)in.cfg.at(key); };

    const int layers = (int)in.attention.size();
    std::vector<dflash_stack_layer> L(layers);
    for (int i = 0; i < layers; ++i) {
        const std::string p = "L" + std::to_string(i) + ".";
        dflash_stack_layer& l = L[i];
        std::memset(&l, 0, sizeof(l));
        l.attention = in.attention[i];
        l.ln = bf(p + "ln");
        l.post_ln = bf(p + "post_ln");
        l.in_proj = qw(p + "in_proj");
        l.out_proj = qw(p + "out_proj");
        l.conv = bf(p + "conv");
        l.a_log = static_cast<const float*>(ptr(p + "a_log"));
        l.dt_bias = static_cast<const float*>(ptr(p + "dt_bias"));
        l.gdn_norm = bf(p + "gdn_norm");
        l.snapshot = static_cast<float*>(ptr(p + "snapshot"));
        l.window = bf(p + "window");
        l.qkv = qw(p + "qkv");
        l.o_proj = qw(p + "o_proj");
        l.q_norm = bf(p + "q_norm");
        l.k_norm = bf(p + "k_norm");
        l.cache_k = bf(p + "cache_k");
        l.cache_v = bf(p + "cache_v");
        l.gate_up = qw(p + "gate_up");
        l.down = qw(p + "down");
    }
    dflash_stack_desc d{};
    d.layers = layers;
    d.hidden = cfg("hidden");
    d.block = cfg("block");
    d.gdn_heads = cfg("gdn_heads");
    d.gdn_key_heads = cfg("gdn_key_heads");
    d.gdn_dk = cfg("gdn_dk");
    d.gdn_dv = cfg("gdn_dv");
    d.conv_kernel = cfg("conv_kernel");
    d.attn_heads = cfg("attn_heads");
    d.kv_heads = cfg("kv_heads");
    d.head_dim = cfg("head_dim");
    d.rotary_dim = cfg("rotary_dim");
    d.max_len = cfg("max_len");
    d.rope_theta = (float)in.cfg.at("rope_theta");
    d.eps = (float)in.cfg.at("eps");
    d.group = cfg("group");
    d.bits = cfg("bits");
    d.rank = 0;
    d.world = 1;
    d.vocab0 = 0;
    d.layer = L.data();
    d.final_norm = bf("final_norm");
    d.lm_head = qw("lm_head");

    dflash_stack* st = nullptr;
    const int context = cfg("context"), keep = cfg("keep"), block = d.block, hidden = d.hidden;
    CHECK(dflash_stack_create(&d, context, &st) == DFLASH_OK);
    if (!st) {
        std::fprintf(stderr, "dflash_stack_create: %s\n", dflash_last_error());
        return 1;
    }
    CHECK(dflash_stack_context(st) == context);
    int32_t *tokens = nullptr, *accepted = nullptr;
    CHECK(cudaMalloc(&tokens, block * sizeof(int32_t)) == cudaSuccess);
    CHECK(cudaMalloc(&accepted, sizeof(int32_t)) == cudaSuccess);
    CHECK(dflash_stack_verify(st, bf("hidden"), static_cast<const int32_t*>(ptr("proposals")), tokens, accepted,
                              nullptr) == DFLASH_OK);
    std::vector<uint16_t> out((size_t)block * hidden);
    std::vector<int32_t> tok(block), acc(1);
    CHECK(cudaMemcpy(out.data(), dflash_stack_output(st), out.size() * 2, cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(cudaMemcpy(tok.data(), tokens, block * 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(cudaMemcpy(acc.data(), accepted, 4, cudaMemcpyDeviceToHost) == cudaSuccess);
    // the forward alone, into a caller buffer, repeats the verify's forward bit for bit
    dflash_bf16* again = nullptr;
    CHECK(cudaMalloc(&again, out.size() * 2) == cudaSuccess);
    CHECK(dflash_stack_forward(st, bf("hidden"), again, nullptr) == DFLASH_OK);
    std::vector<uint16_t> out2(out.size());
    CHECK(cudaMemcpy(out2.data(), again, out2.size() * 2, cudaMemcpyDeviceToHost) == cudaSuccess);
    CHECK(out2 == out);
    // a round with no room left in the caches is refused before any launch
    CHECK(dflash_stack_advance(st, d.max_len) == DFLASH_ERR_INVALID_ARGUMENT);
    CHECK(dflash_stack_commit(st, nullptr, keep, nullptr) == DFLASH_OK);
    CHECK(dflash_stack_advance(st, keep) == DFLASH_OK);
    CHECK(dflash_stack_context(st) == context + keep);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    uint32_t bits = 0;
    CHECK(dflash_device_error(&bits, nullptr) == DFLASH_OK && bits == 0);

    // results: the round's output, tokens, accept count, and every layer's state after it
    std::ofstream rb(dir + "/result.bin", std::ios::binary), rt(dir + "/result.txt");
    size_t off = 0;
    auto put = [&](const std::string& name, const void* host, size_t bytes) {
        rb.write(static_cast<const char*>(host), (std::streamsize)bytes);
        rt << name << " " << off << " " << bytes << "\n";
        off += bytes;
    };
    put("out", out.data(), out.size() * 2);
    put("tokens", tok.data(), tok.size() * 4);
    put("accepted", acc.data(), 4);
    for (int i = 0; i < layers; ++i)
        for (const char* key : {"snapshot", "window", "cache_k", "cache_v"}) {
            const std::string name = "L" + std::to_string(i) + "." + key;
            auto it = in.tensors.find(name);
            if (it == in.tensors.end()) continue;
            std::vector<uint8_t> host(it->second.second);
            CHECK(cudaMemcpy(host.data(), in.base + it->second.first, host.size(), cudaMemcpyDeviceToHost) ==
                  cudaSuccess);
            put(name, host.data(), host.size());
        }
    dflash_stack_destroy(st);
    cudaFree(tokens);
    cudaFree(accepted);
    cudaFree(again);
    cudaFree(in.base);
    return 0;
}

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "cpu";
    int rc = 0;
    try {
        rc = mode == "gpu" ? runGpu() : mode == "stack" ? runStack(argc > 2 ? argv[2] : ".") : runCpu();
    } catch (const std::exception& e) {
        std::fprintf(stderr, "uncaught: %s\n", e.what());
        return 3;
    }
    std::printf("%s: %d checks, %d failures\n", mode.c_str(), g_checks, g_failures);
    return rc ? rc : (g_failures ? 1 : 0);
}
