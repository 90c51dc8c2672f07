// The C++ surface on a B200: denoise through one CUDA graph equals the step-by-step observer path and
// the recovery wrapper (allocation failure injected before step 2) bit-exactly; run_dit and layer
// wrappers keep the reference contracts.
#include "ernie_b200/ernie.h"
#include "ernie_synth.h"
#include <cmath>
#include <iostream>

using namespace ernie;

static int failures = 0;
#define REQUIRE(cond, msg)                                                                                          \
    do                                                                                                              \
    {                                                                                                               \
        if (!(cond))                                                                                                \
        {                                                                                                           \
            std::cerr << "FAILED: " << msg << " line " << __LINE__ << "\n";                                        \
            ++failures;                                                                                             \
        }                                                                                                           \
    } while (0)

static Tensor normal(int w, int h, int c, uint64_t stream)
{
    Tensor t = c > 1 ? Tensor(w, h, c) : Tensor(w, h);
    for (size_t i = 0; i < t.total(); ++i) t[i] = float(ernie_synth_normal(21, stream, i));
    return t;
}

int main()
{
    try
    {
        GpuContext ctx(true, 0);
        DitModel model(ctx, 2);
        model.synthesize(11);
        const int w = 8, h = 6, text = 16, valid = 10;
        auto k = dit_constants({}, w, h, valid, text);
        Tensor txt = pad_text(normal(3072, valid, 1, ERNIE_SYNTH_TEXT), text);
        const std::vector<Tensor> constants{txt, k[0], k[1], k[2]};
        const Tensor initial = normal(w, h, 128, ERNIE_SYNTH_LATENT);

        DenoiseSession session(model, w, h, text, valid, Precision::BF16);
        session.set_constants(constants);
        std::vector<DenoiseStepStats> stats;
        const Tensor graph = denoise(session, initial, 8, stats);
        REQUIRE(stats.size() == 8 && stats.back().complete, "graph denoise stats");
        size_t observed = 0;
        const Tensor stepped = denoise(session, initial, 8, stats,
                                       [&](size_t i, const Tensor &pred, const Tensor &latent) {
                                           REQUIRE(i == observed && pred.total() == latent.total(), "observer order");
                                           ++observed;
                                       });
        REQUIRE(observed == 8 && graph.data == stepped.data, "graph and observer paths differ");

        CudaDenoiseBackend backend(model, w, h, text, valid, Precision::BF16, constants);
        CudaDenoiseSettings settings;
        settings.before_step = [](unsigned attempt, int step) {
            if (attempt == 0 && step == 2) throw GpuAllocationError("controlled allocation failure");
        };
        CudaDenoiseStats rstats;
        const Tensor recovered = denoise_with_recovery(backend, initial, 8, 0, settings, rstats);
        REQUIRE(recovered.data == graph.data && rstats.retries == 1 && rstats.query_rows == 64 &&
                    attention_query_rows(ctx) == 64,
                "recovery changed bits or bounds");

        DeviceTensor dlat = DeviceTensor::upload(ctx, initial);
        DitStats dstats;
        const Tensor prediction = run_dit(session, dlat, 923.0769f, dstats).download();
        bool finite = true;
        for (float v : prediction.data) finite = finite && std::isfinite(v);
        REQUIRE(finite && prediction.total() == initial.total(), "run_dit prediction");
        REQUIRE(finite_latent(ctx, dlat), "finite_latent");

        Tensor x(64, 4);
        DeviceTensor dx = DeviceTensor::upload(ctx, x);
        bool threw = false;
        try
        {
            rms_norm(ctx, dx, Tensor(64));
        }
        catch (const std::invalid_argument &)
        {
            threw = true;
        }
        REQUIRE(threw, "RMSNorm width 64 accepted");
        threw = false;
        try
        {
            set_attention_query_rows(ctx, 48);
        }
        catch (const std::invalid_argument &)
        {
            threw = true;
        }
        REQUIRE(threw, "query rows 48 accepted");
    }
    catch (const std::exception &e)
    {
        std::cerr << "exception: " << e.what() << "\n";
        return 1;
    }
    if (failures) return 1;
    std::cout << "host GPU contracts passed\n";
    return 0;
}
