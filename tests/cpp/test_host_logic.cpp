// Host-side contracts of the C++ surface (no GPU): schedule, features, constants, text padding, error
// mapping, weight placement decisions, weight-session admission/leases and the recovery loop with a
// host-side fake backend. Cases follow the reference's tests/test_latent_contract.cpp,
// tests/test_weight_placement.cpp:38-78, tests/test_weight_session.cpp:36-131 and
// tests/test_memory_execution.cpp:298-419 (recovery_contract); tensor files as src/tensor_io.cpp:10-43.
#include "ernie_b200/ernie.h"
#include <cmath>
#include <filesystem>
#include <fstream>
#include <cstdio>
#include <cstdlib>
#include <iostream>
#include <limits>
#include <memory>
#include <new>
#include <tuple>
#include <unistd.h>

using namespace ernie;

static int failures = 0;
#define REQUIRE(cond, msg)                                                                                          \
    do                                                                                                              \
    {                                                                                                               \
        if (!(cond))                                                                                                \
        {                                                                                                           \
            std::cerr << "FAILED: " << msg << " (" << #cond << ") line " << __LINE__ << "\n";                     \
            ++failures;                                                                                             \
        }                                                                                                           \
    } while (0)

template <class E, class F> bool throws(F &&f)
{
    try
    {
        f();
    }
    catch (const E &)
    {
        return true;
    }
    catch (...)
    {
        return false;
    }
    return false;
}

static void latent_contract()
{
    REQUIRE(throws<std::invalid_argument>([] { FlowSchedule::turbo(0); }), "steps 0 accepted");
    REQUIRE(throws<std::invalid_argument>([] { FlowSchedule::turbo(1001); }), "steps 1001 accepted");
    const auto s = FlowSchedule::turbo();
    REQUIRE(throws<std::out_of_range>([&] { s.delta(8); }), "exhausted schedule accepted");
    REQUIRE(s.sigmas.front() == 1.f && s.sigmas.back() == 0.f, "schedule endpoints");
    for (size_t i = 0; i < 8; ++i) REQUIRE(s.delta(i) < 0.f, "schedule does not descend");
    REQUIRE(s.timesteps[0] == 1000.f, "first timestep");
    const auto lin = FlowSchedule::linear(4);
    REQUIRE(lin.sigmas[1] == 0.75f && lin.sigmas[4] == 0.f, "linear schedule");
    REQUIRE(throws<std::invalid_argument>([] { timestep_features(1000.5f); }), "timestep above 1000 accepted");
    const Tensor f = timestep_features(0.f);
    REQUIRE(f.total() == 4096 && f[0] == 0.f && f[2048] == 1.f, "features of t=0 are sin 0 / cos 1");
}

static void conditioning_contract()
{
    const auto k = dit_constants({}, 4, 3, 5, 8);
    REQUIRE(k.size() == 3 && k[0].total() == 20 * 128 && k[2].total() == 20, "constant shapes");
    REQUIRE(k[2][16] == 0.f && k[2][17] == -1e30f, "mask hides slots past the valid text");
    REQUIRE(throws<std::invalid_argument>([] { dit_constants({}, 4, 3, 9, 8); }), "valid > bucket accepted");
    REQUIRE(throws<std::invalid_argument>([] { dit_constants({}, 64, 65, 64, 2048, 6144); }), "static limit");
    std::vector<float> bad(64, 1.f);
    bad[5] = 0.f;
    REQUIRE(throws<std::invalid_argument>([&] { dit_constants(bad, 2, 2, 1, 1); }), "non-positive frequency accepted");
    Tensor text(3072, 3);
    for (auto &v : text.data) v = 2.f;
    const Tensor padded = pad_text(text, 8);
    REQUIRE(padded.h == 8 && padded[3072 * 3 - 1] == 2.f && padded[3072 * 3] == 0.f, "pad_text zero fill");
    REQUIRE(throws<std::invalid_argument>([&] { pad_text(text, 2); }), "bucket smaller than text accepted");
}

static void error_mapping()
{
    REQUIRE(throws<GpuAllocationError>([] { check_cuda(ERNIE_CUDA_OUT_OF_MEMORY, "x"); }), "-100 must map to OOM");
    REQUIRE(throws<std::runtime_error>([] { check_cuda(ERNIE_CUDA_ERROR, "x"); }) &&
                !throws<GpuAllocationError>([] { check_cuda(ERNIE_CUDA_ERROR, "x"); }),
            "-1 must not be OOM");
    GpuContext disabled(false, -1, false);
    REQUIRE(!disabled.available() && !disabled.initialization_error().empty(), "disabled context");
    REQUIRE(throws<std::logic_error>([&] { disabled.handle(); }), "handle of an unavailable context");
}

static void placement_contract()
{
    auto decision = [](std::uint64_t budget, std::uint64_t usage) {
        return choose_weight_placement(WeightMemory::Auto, false, 100, 20, DeviceMemoryBudget{budget, usage});
    };
    REQUIRE(!decision(200, 80).host, "Exact budget boundary must fit");
    REQUIRE(decision(200, 81).host, "Budget usage was not subtracted");
    REQUIRE(decision(200, 201).available_bytes == 0u && decision(200, 201).host, "Over-budget usage wrapped");
    REQUIRE(choose_weight_placement(WeightMemory::Auto, false, UINT64_MAX, UINT64_MAX, DeviceMemoryBudget{10, 0}).host,
            "reserve larger than budget");
    REQUIRE(std::string(choose_weight_placement(WeightMemory::Auto, true, 1, 0, DeviceMemoryBudget{1000, 0}).reason) ==
                "shape",
            "shape preference");
    const auto absent = choose_weight_placement(WeightMemory::Auto, false, 100, 20, std::nullopt);
    REQUIRE(!absent.host && !absent.available_bytes && std::string(absent.reason) == "unavailable", "missing budget");
    REQUIRE(choose_weight_placement(WeightMemory::Host, false, 1, 0, std::nullopt).host, "explicit host");
    REQUIRE(!choose_weight_placement(WeightMemory::Device, true, 100, 20, DeviceMemoryBudget{1, 0}).host,
            "explicit device");
    int queries = 0;
    std::uint64_t usage = 0;
    WeightPlacement dynamic(WeightMemory::Auto, 20, [&]() -> std::optional<DeviceMemoryBudget> {
        ++queries;
        return DeviceMemoryBudget{200, usage};
    });
    const bool first = dynamic.use_host("block-00", 100, false);
    usage = 81;
    const bool second = dynamic.use_host("block-01", 100, false);
    usage = 0;
    const bool third = dynamic.use_host("block-02", 100, false);
    REQUIRE(!first && second && !third && queries == 3 && dynamic.host_requests() == 1 &&
                dynamic.device_requests() == 2,
            "dynamic budget queries");
    WeightPlacement manual(WeightMemory::Host, 0, []() -> std::optional<DeviceMemoryBudget> {
        throw std::runtime_error("an explicit mode must not read the device budget");
    });
    REQUIRE(manual.use_host("block", 100, false) && manual.host_requests() == 1, "explicit mode read the budget");
    std::string seen_reason;
    WeightPlacement cached(WeightMemory::Auto, 20, [] { return std::optional<DeviceMemoryBudget>(DeviceMemoryBudget{1000, 0}); },
                           [&](const std::string &, const WeightPlacementDecision &d) { seen_reason = d.reason; });
    REQUIRE(cached.use_host("block", 100, false, true, "prefetch") && seen_reason == "prefetch",
            "cache preference in auto mode");
    WeightPlacement unavailable(WeightMemory::Auto, 20);
    REQUIRE(!unavailable.use_host("block", 100, false) && unavailable.unavailable_queries() == 1, "unavailable reader");
    REQUIRE(parse_weight_memory("host") == WeightMemory::Host &&
                throws<std::invalid_argument>([] { parse_weight_memory("gpu"); }),
            "parse_weight_memory");
}

static int live_payloads = 0;
struct FakePayload
{
    FakePayload() { ++live_payloads; }
    ~FakePayload() { --live_payloads; }
};
static WeightSession::Payload fake_payload() { return std::make_shared<FakePayload>(); }

static void session_contract()
{
    int request, other_request;
    std::uint64_t available = 1000;
    auto inspect = [](const WeightSession::Payload &) -> std::optional<std::uint64_t> { return 10; };
    auto reader = [&]() -> std::optional<std::uint64_t> { return available; };
    {
        WeightSession session({20, 30}, reader, inspect);
        int requested_cache = 0, loaded = 0;
        auto load = [&](bool cache) {
            ++loaded;
            requested_cache += cache;
            return fake_payload();
        };
        // a repeated sequential scan hits the admitted prefix although the sequence exceeds capacity
        for (int step = 0; step < 3; ++step)
            for (std::size_t block = 0; block < 3; ++block)
            {
                auto lease = session.acquire(block, "graph", &request, 10, load);
                REQUIRE(live_payloads <= 3 && session.stats().live_bytes <= 20, "Unbounded resident weights");
                lease.complete();
            }
        REQUIRE(loaded == 5 && requested_cache == 2 && session.stats().hits == 4 && session.stats().peak_bytes == 20 &&
                    live_payloads == 2,
                "Cache scan thrashed or accounting differs");
        REQUIRE(throws<std::logic_error>([&] { session.acquire(0, "changed", &request, 10, load); }), "identity change");
        REQUIRE(throws<std::logic_error>([&] { session.acquire(0, "graph", &other_request, 10, load); }), "request change");
        {
            auto lease = session.acquire(0, "graph", &request, 10, load);
            REQUIRE(throws<std::logic_error>([&] { session.acquire(1, "graph", &request, 10, load); }),
                    "second concurrent lease");
            session.cancel();
            REQUIRE(live_payloads == 1 && session.stats().live_bytes == 10, "Cancel released an active payload");
        }
        REQUIRE(live_payloads == 0 && session.stats().live_bytes == 0, "Cancelled lease leaked");
        REQUIRE(throws<std::logic_error>([&] { session.acquire(0, "graph", &request, 10, load); }), "cancelled session");
    }
    {
        WeightSession pressure({20, 30}, reader, inspect);
        auto load = [](bool) { return fake_payload(); };
        auto first = pressure.acquire(0, "graph", &request, 10, load);
        first.complete();
        available = 35;
        auto second = pressure.acquire(1, "graph", &request, 10, load);
        REQUIRE(!second.cached() && pressure.stats().evictions == 1 && live_payloads == 1,
                "Pressure failed to evict idle weights");
        available = 1000;
    }
    {
        // enough RAM above the reserve to reuse a cached block but not to load another: the hit must not
        // reserve a second copy; below the reserve the idle block is dropped and reloaded
        WeightSession hit({20, 30}, reader, inspect);
        auto load = [](bool) { return fake_payload(); };
        auto first = hit.acquire(0, "graph", &request, 10, load);
        first.complete();
        available = 35;
        auto same = hit.acquire(0, "graph", &request, 10, load);
        REQUIRE(same.cached() && hit.stats().hits == 1 && hit.stats().loads == 1 && hit.stats().evictions == 0,
                "Cache hit reserved a second copy of its weights");
        same.complete();
        available = 29;
        auto pressured = hit.acquire(0, "graph", &request, 10, load);
        REQUIRE(!pressured.cached() && hit.stats().evictions == 1 && hit.stats().loads == 2,
                "Cache hit ignored the RAM reserve under pressure");
        pressured.complete();
        available = 1000;
    }
    {
        WeightSession moves({20, 30}, reader, inspect);
        auto lease = moves.acquire(0, "graph", &request, 10, [](bool) { return fake_payload(); });
        auto moved = std::move(lease);
        REQUIRE(throws<std::logic_error>([&] { lease.payload(); }), "moved-from lease still holds the payload");
        REQUIRE(moved.payload() != nullptr && moved.cached(), "moved lease lost the payload");
        moved.complete();
        REQUIRE(moves.contains(0) && live_payloads == 1, "completed lease did not return to the cache");
    }
    REQUIRE(live_payloads == 0, "destroyed session kept an idle payload");
    {
        WeightSession oversized({20, 30}, reader, [](const WeightSession::Payload &) -> std::optional<std::uint64_t> { return 21; });
        auto lease = oversized.acquire(0, "graph", &request, 10, [](bool) { return fake_payload(); });
        REQUIRE(!lease.cached() && oversized.stats().live_bytes == 0, "Measured charge exceeded budget");
    }
    {
        WeightSession unmeasured({20, 30}, reader,
                                 [](const WeightSession::Payload &) -> std::optional<std::uint64_t> { return std::nullopt; });
        auto lease = unmeasured.acquire(0, "graph", &request, 10, [](bool) { return fake_payload(); });
        REQUIRE(!lease.cached(), "Unverified payload entered the cache");
    }
    {
        WeightSession::Lease orphan;
        {
            WeightSession owner({20, 30}, reader, inspect);
            orphan = owner.acquire(0, "graph", &request, 10, [](bool) { return fake_payload(); });
        }
        REQUIRE(live_payloads == 1, "Session destruction invalidated an active lease");
        orphan.complete();
        REQUIRE(live_payloads == 0, "Session destruction leaked a payload");
    }
    {
        WeightSession failure({20, 30}, reader, inspect);
        REQUIRE(throws<std::runtime_error>([&] {
                    failure.acquire(0, "graph", &request, 10,
                                    [](bool) -> WeightSession::Payload { throw std::runtime_error("read failure"); });
                }),
                "loader failure propagates");
        auto lease = failure.acquire(0, "graph", &request, 10, [](bool) { return fake_payload(); });
        REQUIRE(live_payloads == 1, "Load failure poisoned session");
    }
    REQUIRE(live_payloads == 0, "Abandoned lease leaked");
    {
        WeightSession no_budget({20, 30}, [] { return std::optional<std::uint64_t>(); }, inspect);
        auto lease = no_budget.acquire(0, "graph", &request, 10, [](bool) { return fake_payload(); });
        REQUIRE(!lease.cached() && no_budget.stats().unavailable_queries, "Missing budget fabricated admission");
    }
}

// Host-side fake of the reference's tiny denoiser (v = 0.125 x), with a controllable allocation failure.
class TinyBackend : public DenoiseBackend
{
  public:
    Tensor current;
    std::vector<std::tuple<unsigned, int>> begun;
    void begin_attempt(unsigned attempt, const Tensor &checkpoint, int) override
    {
        begun.emplace_back(attempt, 0);
        current = checkpoint;
    }
    Tensor run_step(int, float, float delta) override
    {
        Tensor prediction = current;
        for (auto &v : prediction.data) v *= 0.125f;
        for (size_t i = 0; i < current.total(); ++i)
        {
            const float change = delta * prediction[i];
            current[i] = current[i] + change;
        }
        return prediction;
    }
    Tensor latent() override { return current; }
    void end_attempt() override {}
};

static bool exact(const Tensor &a, const Tensor &b) { return a.data == b.data; }

static void recovery_contract()
{
    Tensor initial(3, 2, 128);
    for (size_t i = 0; i < initial.total(); ++i) initial[i] = float(int(i % 17) - 8) / 4.f;
    constexpr int steps = 4;
    const auto schedule = FlowSchedule::turbo(steps);
    CudaDenoiseSettings base;
    TinyBackend backend;
    CudaDenoiseStats baseline_stats;
    std::vector<Tensor> checkpoints;
    CudaDenoiseObservers baseline_observer;
    baseline_observer.step = [&](size_t index, const Tensor &, const Tensor &value, const DenoiseStepStats &st) {
        REQUIRE(index == checkpoints.size() && st.complete && st.timestep == schedule.timesteps[index] &&
                    st.delta == schedule.delta(index),
                "Baseline schedule or checkpoint differs");
        checkpoints.push_back(value);
    };
    const Tensor baseline = denoise_with_recovery(backend, initial, steps, 0, base, baseline_stats, baseline_observer);
    REQUIRE(checkpoints.size() == steps && baseline_stats.retries == 0 && baseline_stats.query_rows == 128 &&
                !exact(baseline, initial),
            "Tiny model did not execute real denoising");
    for (int c = 0; c < 128; ++c)
    {
        float expected = initial[size_t(c) * 6];
        for (int i = 0; i < steps; ++i) expected += schedule.delta(i) * (expected * 0.125f);
        REQUIRE(std::abs(baseline[size_t(c) * 6] - expected) <= 3e-7f, "Tiny denoiser differs from independent Euler");
    }
    std::vector<std::pair<unsigned, int>> attempted;
    std::vector<size_t> committed;
    std::vector<std::tuple<unsigned, int, int>> retries;
    CudaDenoiseSettings injected;
    injected.before_step = [&](unsigned attempt, int step) {
        attempted.emplace_back(attempt, step);
        if (attempt == 0 && step == 2) throw GpuAllocationError("controlled allocation failure after step 1");
    };
    CudaDenoiseObservers observer;
    observer.retry = [&](unsigned attempt, int step, int rows, const std::string &) {
        retries.emplace_back(attempt, step, rows);
    };
    observer.step = [&](size_t index, const Tensor &, const Tensor &value, const DenoiseStepStats &) {
        committed.push_back(index);
        REQUIRE(exact(value, checkpoints.at(index)), "Recovery changed a completed latent");
    };
    CudaDenoiseStats recovered;
    REQUIRE(exact(denoise_with_recovery(backend, initial, steps, 0, injected, recovered, observer), baseline),
            "Allocation recovery changed final tensor bits");
    REQUIRE((attempted == std::vector<std::pair<unsigned, int>>{{0, 0}, {0, 1}, {0, 2}, {1, 2}, {1, 3}}) &&
                (committed == std::vector<size_t>{0, 1, 2, 3}) &&
                (retries == std::vector<std::tuple<unsigned, int, int>>{{1, 2, 64}}) && recovered.retries == 1 &&
                recovered.query_rows == 64,
            "Recovery repeated a committed step or failed to shrink chunks");
    attempted.clear();
    committed.clear();
    injected.before_step = [&](unsigned attempt, int step) {
        attempted.emplace_back(attempt, step);
        if (!attempt && step == 3) throw std::bad_alloc();
    };
    CudaDenoiseStats resumed;
    REQUIRE(exact(denoise_with_recovery(backend, checkpoints[1], steps, 2, injected, resumed, observer), baseline),
            "Nonzero start-step recovery changed output");
    REQUIRE((attempted == std::vector<std::pair<unsigned, int>>{{0, 2}, {0, 3}, {1, 3}}) &&
                (committed == std::vector<size_t>{2, 3}) && resumed.retries == 1,
            "Nonzero start-step recovery renumbered or replayed the schedule");
    for (unsigned limit : {0u, 3u})
    {
        CudaDenoiseSettings bounded;
        bounded.retries = limit;
        unsigned calls = 0;
        bounded.before_step = [&](unsigned attempt, int step) {
            REQUIRE(attempt == calls++ && step == 0, "Failed restart changed checkpoint or attempt index");
            throw GpuAllocationError("persistent controlled failure");
        };
        CudaDenoiseStats exhausted;
        std::string message;
        try
        {
            denoise_with_recovery(backend, initial, steps, 0, bounded, exhausted);
        }
        catch (const GpuAllocationError &e)
        {
            message = e.what();
        }
        REQUIRE(calls == limit + 1 && exhausted.retries == limit && exhausted.query_rows == int(128 >> limit) &&
                    message.find("exhausted") != std::string::npos,
                "Recovery exceeded its retry/chunk bounds");
    }
    CudaDenoiseSettings fatal;
    unsigned calls = 0;
    fatal.before_step = [&](unsigned, int) {
        ++calls;
        check_cuda(ERNIE_CUDA_ERROR, "injected generic failure");
    };
    CudaDenoiseStats fatal_stats;
    bool ordinary = false;
    try
    {
        denoise_with_recovery(backend, initial, steps, 0, fatal, fatal_stats);
    }
    catch (const GpuAllocationError &)
    {
    }
    catch (const std::runtime_error &)
    {
        ordinary = true;
    }
    REQUIRE(ordinary && calls == 1 && fatal_stats.retries == 0, "Fatal computation error was retried");
    CudaDenoiseSettings too_many;
    too_many.retries = 4;
    CudaDenoiseStats s;
    REQUIRE(throws<std::invalid_argument>([&] { denoise_with_recovery(backend, initial, steps, 0, too_many, s); }),
            "more than three retries accepted");
}

static void tensor_io_contract()
{
    const auto dir = std::filesystem::temp_directory_path() / ("ernie_b200_io_" + std::to_string(::getpid()));
    std::filesystem::remove_all(dir);
    std::filesystem::create_directories(dir);
    const std::string path = (dir / "t.f32").string();
    Tensor t(3, 2, 2);
    for (size_t i = 0; i < t.total(); ++i) t[i] = float(i) - 2.5f;
    write_tensor(path, t);
    REQUIRE(std::filesystem::file_size(path) == 48, "raw FP32 size");
    const Tensor back = read_tensor(path, 3, 2, 2);
    REQUIRE(back.data == t.data && back.w == 3 && back.h == 2 && back.c == 2, "round trip");
    REQUIRE(throws<std::runtime_error>([&] { write_tensor(path, t); }), "existing trace file overwritten");
    REQUIRE(throws<std::runtime_error>([&] { read_tensor(path, 4, 2, 2); }), "wrong size accepted");
    {
        std::ofstream f((dir / "nan.f32").string(), std::ios::binary);
        const float v[2] = {1.f, NAN};
        f.write(reinterpret_cast<const char *>(v), sizeof(v));
    }
    REQUIRE(throws<std::runtime_error>([&] { read_tensor((dir / "nan.f32").string(), 2); }), "non-finite accepted");
    REQUIRE(numbered("block-", 7) == "block-07" && numbered("block-", 35) == "block-35", "numbered");
    std::filesystem::remove_all(dir);
    const Tensor n1 = initial_noise(5, 4, 42), n2 = initial_noise(5, 4, 42), n3 = initial_noise(5, 4, 43);
    REQUIRE(n1.c == 128 && n1.h == 4 && n1.w == 5 && n1.data == n2.data && n1.data != n3.data, "initial noise");
    REQUIRE(throws<std::invalid_argument>([] { initial_noise(0, 4, 1); }), "empty latent accepted");
}

// tests/test_img2img_contract.cpp: endpoints, interpolation, round-half-up step selection, rejections
static void img2img_contract()
{
    const FlowSchedule schedule = FlowSchedule::turbo(8);
    Tensor encoded(2, 3, 128), noise(2, 3, 128);
    for (auto &v : encoded.data) v = 2.f;
    for (auto &v : noise.data) v = -1.f;
    const Img2ImgStart zero = make_img2img_start(encoded, Tensor(), schedule, 0.f, 1);
    REQUIRE(zero.start_step == 8 && zero.denoise_steps == 0 && zero.sigma == 0.f && zero.latent.data == encoded.data,
            "strength zero");
    const Img2ImgStart one = make_img2img_start(encoded, noise, schedule, 1.f, 1);
    REQUIRE(one.start_step == 0 && one.denoise_steps == 8 && one.sigma == 1.f && one.latent.data == noise.data,
            "strength one");
    for (const float fraction : {.25f, .5f, .75f})
    {
        const int count = int(fraction * 8);
        const Img2ImgStart start = make_img2img_start(encoded, noise, schedule, fraction, 1);
        const float expected = -start.sigma + (1.f - start.sigma) * 2.f;
        bool same = start.denoise_steps == count && start.start_step == 8 - count;
        for (float v : start.latent.data) same = same && v == expected;
        REQUIRE(same, "strength step selection / interpolation");
    }
    REQUIRE(make_img2img_start(encoded, noise, schedule, .3125f, 1).denoise_steps == 3, "half step rounds up");
    REQUIRE(make_img2img_start(encoded, noise, schedule, std::numeric_limits<float>::min(), 1).denoise_steps == 1,
            "positive strength skipped all steps");
    for (const float bad : {-1.f, 1.01f, INFINITY, NAN})
        REQUIRE(throws<std::invalid_argument>([&] { make_img2img_start(encoded, noise, schedule, bad); }),
                "bad strength accepted");
    REQUIRE(throws<std::invalid_argument>([&] { make_img2img_start(encoded, noise, schedule, .5f, 0); }),
            "zero threads accepted");
    REQUIRE(throws<std::invalid_argument>([&] { make_img2img_start(encoded, Tensor(1, 1, 128), schedule, .5f); }),
            "mismatched noise accepted");
    FlowSchedule malformed = schedule;
    malformed.sigmas[4] = NAN;
    REQUIRE(throws<std::invalid_argument>([&] { make_img2img_start(encoded, noise, malformed, .5f); }),
            "NaN sigma accepted");
    malformed = schedule;
    malformed.timesteps.pop_back();
    REQUIRE(throws<std::invalid_argument>([&] { make_img2img_start(encoded, noise, malformed, .5f); }),
            "short schedule accepted");
    noise[6] = NAN; // channel 1, element 0
    REQUIRE(throws<std::invalid_argument>([&] { make_img2img_start(encoded, noise, schedule, .5f); }),
            "NaN noise accepted");
}

// rgb_image (src/pipeline.cpp:145-163) and the VAE decoder's tensor table (no device needed)
static void vae_contract()
{
    Tensor decoded(4, 1, 3);
    const float values[4] = {-3.f, 0.f, 0.5f, 1.f / 255.f};
    for (int c = 0; c < 3; ++c)
        for (int i = 0; i < 4; ++i) decoded[size_t(c) * 4 + size_t(i)] = values[i] * float(c + 1);
    const RgbImage image = rgb_image(decoded);
    REQUIRE(image.width == 4 && image.height == 1 && image.pixels.size() == 12, "RGB shape");
    // channel 0: -3 -> 0, 0 -> 128 (127.5 rounds to even), 0.5 -> 191, 1/255 -> 128
    const uint8_t expected0[4] = {0, 128, 191, 128};
    for (int i = 0; i < 4; ++i) REQUIRE(image.pixels[size_t(i) * 3] == expected0[i], "RGB byte " << i);
    REQUIRE(image.pixels[2 * 3 + 2] == 255, "0.5 * 3 clamps to 255");
    decoded[5] = std::numeric_limits<float>::quiet_NaN();
    REQUIRE(throws<std::runtime_error>([&] { rgb_image(decoded); }), "non-finite pixel accepted");
    REQUIRE(throws<std::runtime_error>([&] { rgb_image(Tensor(4, 1, 4)); }), "4 channels accepted");
    const auto tensors = VaeDecoder::tensors();
    REQUIRE(tensors.size() == 140, "VAE tensor count " << tensors.size());
    REQUIRE(tensors.front().first == "post_quant_conv.weight" && tensors.back().first == "decoder.conv_out.bias",
            "VAE tensor order");
    size_t params = 0;
    for (const auto &t : tensors)
    {
        size_t n = 1;
        for (int d : t.second) n *= size_t(d);
        params += n;
    }
    REQUIRE(params == 49620259, "VAE parameter count " << params);
    const auto enc = VaeEncoder::tensors();
    REQUIRE(enc.size() == 110, "VAE encoder tensor count " << enc.size());
    REQUIRE(enc.front().first == "encoder.conv_in.weight" && enc.front().second == std::vector<int>({128, 3, 3, 3}) &&
                enc.back().first == "bn.running_var",
            "VAE encoder tensor order");
    size_t enc_params = 0;
    for (const auto &t : enc)
    {
        size_t n = 1;
        for (int d : t.second) n *= size_t(d);
        enc_params += n;
    }
    REQUIRE(enc_params == 34426112, "VAE encoder parameter count " << enc_params);
}

// sample_pe_token (src/prompt_enhancer.cpp:33-66) with the cases of the reference's sampling test
// (tests/test_pe_sampling.cpp:24-100): greedy ties, top-p truncation, frequencies, reproducibility, options
static void pe_sampling_contract()
{
    PeOptions options;
    std::mt19937 first(42), second(42);
    options.greedy = true;
    REQUIRE(sample_pe_token({-1.f, 4.f, 4.f}, options, first) == 1, "greedy tie must choose the first token");
    options.greedy = false;
    options.temperature = 1;
    options.top_p = .6f;
    const std::vector<float> dist = {std::log(.7f), std::log(.2f), std::log(.1f)};
    for (int i = 0; i < 32; ++i) REQUIRE(sample_pe_token(dist, options, first) == 0, "top-p 0.6 keeps only the 0.7 token");
    options.top_p = 1;
    first.seed(20260906);
    int counts[3] = {0, 0, 0};
    constexpr int draws = 100000;
    for (int i = 0; i < draws; ++i) ++counts[sample_pe_token(dist, options, first)];
    const double expected[3] = {.7, .2, .1};
    for (int i = 0; i < 3; ++i)
        REQUIRE(std::abs(double(counts[i]) / draws - expected[i]) <= .01, "sampling frequency " << i);
    first.seed(42);
    second.seed(42);
    for (int i = 0; i < 32; ++i)
        REQUIRE(sample_pe_token({-1.f, 4.f, 4.f}, options, first) == sample_pe_token({-1.f, 4.f, 4.f}, options, second),
                "sampling must be reproducible");
    for (float bad : {0.f, -1.f, INFINITY, NAN})
    {
        options.temperature = bad;
        REQUIRE(throws<std::invalid_argument>([&] { sample_pe_token(dist, options, first); }), "temperature " << bad);
    }
    options.temperature = 1;
    for (float bad : {0.f, -1.f, 1.01f, INFINITY, NAN})
    {
        options.top_p = bad;
        REQUIRE(throws<std::invalid_argument>([&] { sample_pe_token(dist, options, first); }), "top-p " << bad);
    }
    options.top_p = 1;
    for (int bad : {0, -1, 2049})
    {
        options.max_tokens = bad;
        REQUIRE(throws<std::invalid_argument>([&] { sample_pe_token(dist, options, first); }), "max tokens " << bad);
    }
    options.max_tokens = 8;
    REQUIRE(throws<std::invalid_argument>([&] { sample_pe_token({}, options, first); }), "empty logits accepted");
    REQUIRE(throws<std::runtime_error>([&] { sample_pe_token({0.f, NAN}, options, first); }), "NaN logits accepted");
}

// text_constants and text_embeddings (src/text_encoder.cpp:48-104) without a device
static void text_contract()
{
    std::vector<float> f(64);
    for (int j = 0; j < 64; ++j) f[size_t(j)] = 1.f / std::pow(1000000.f, float(j) / 64.f);
    const auto k = text_constants(f, 5);
    REQUIRE(k.size() == 3 && k[0].w == 128 && k[0].h == 5 && k[2].w == 5 && k[2].h == 5, "text constant shapes");
    REQUIRE(k[0][128 * 3 + 7] == std::cos(3.f * f[7]) && k[0][128 * 3 + 71] == k[0][128 * 3 + 7], "cos row");
    REQUIRE(k[1][128 * 4 + 63] == std::sin(4.f * f[63]), "sin row");
    REQUIRE(k[2][1 * 5 + 1] == 0.f && k[2][1 * 5 + 2] == -std::numeric_limits<float>::max(), "causal mask");
    REQUIRE(throws<std::invalid_argument>([&] { text_constants(f, 2049); }), "bucket 2049 accepted");
    f[3] = -1.f;
    REQUIRE(throws<std::invalid_argument>([&] { text_constants(f, 4); }), "negative frequency accepted");
    REQUIRE(throws<std::invalid_argument>([&] { text_embeddings("/nonexistent/embeddings.bf16", {1, 2}, 4); }),
            "missing table accepted");
    REQUIRE(throws<std::invalid_argument>([&] { text_embeddings("/nonexistent/embeddings.bf16", {1, 2, 3}, 2); }),
            "more ids than the bucket accepted");
}

int main()
{
    latent_contract();
    vae_contract();
    text_contract();
    conditioning_contract();
    error_mapping();
    placement_contract();
    session_contract();
    recovery_contract();
    tensor_io_contract();
    img2img_contract();
    pe_sampling_contract();
    if (failures)
    {
        std::cerr << failures << " host contract failure(s)\n";
        return 1;
    }
    std::cout << "host contracts passed\n";
    return 0;
}
