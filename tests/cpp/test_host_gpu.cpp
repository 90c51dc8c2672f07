// The C++ surface on a B200: denoise through one CUDA graph equals the step-by-step observer path and
// the recovery wrapper (allocation failure injected before step 2) bit-exactly; run_dit and layer
// wrappers keep the reference contracts; the pipeline's DiT stage (seeded noise, constants, graph or
// traced path) equals the same denoise built by hand and writes the reference's trace files.
#include "ernie_b200/ernie.h"
#include "ernie_synth.h"
#include <cmath>
#include <filesystem>
#include <fstream>
#include <iostream>
#include <unistd.h>

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

        // DiT stage: 128x96 pixels -> 8x6 latent, 10 prompt tokens in a 16-slot bucket, seed 3
        {
            DitStageRequest req;
            req.width = 128;
            req.height = 96;
            req.seed = 3;
            const Tensor prompt = normal(3072, 10, 1, ERNIE_SYNTH_TEXT);
            int notified = 0;
            const DitStageResult fast =
                run_dit_stage(model, prompt, 16, {}, req, [&](const DitStageProgress &p) { notified += p.stage == "denoise"; });
            auto kk = dit_constants({}, 8, 6, 10, 16);
            DenoiseSession manual(model, 8, 6, 16, 10, Precision::BF16);
            manual.set_constants({pad_text(prompt, 16), kk[0], kk[1], kk[2]});
            std::vector<DenoiseStepStats> mstats;
            const Tensor by_hand = denoise(manual, initial_noise(8, 6, 3), 8, mstats);
            REQUIRE(fast.latent.data == by_hand.data && fast.steps.size() == 8 && notified == 8,
                    "DiT stage differs from the hand-built denoise");
            const auto dir = std::filesystem::temp_directory_path() / ("ernie_trace_" + std::to_string(::getpid()));
            std::filesystem::remove_all(dir);
            std::filesystem::create_directories(dir);
            req.trace = dir.string();
            const DitStageResult traced = run_dit_stage(model, prompt, 16, {}, req);
            REQUIRE(traced.latent.data == fast.latent.data, "traced DiT stage differs from the graph path");
            bool files = true;
            for (int i = 0; i < 8; ++i)
                files = files && std::filesystem::file_size(dir / ("prediction-" + std::to_string(i) + ".f32")) ==
                                     size_t(128 * 8 * 6 * 4) &&
                        std::filesystem::file_size(dir / ("step-" + std::to_string(i) + ".f32")) == size_t(128 * 8 * 6 * 4);
            REQUIRE(files, "trace files");
            const Tensor last = read_tensor((dir / "step-7.f32").string(), 8, 6, 128);
            REQUIRE(last.data == traced.latent.data, "last traced step is the result");
            bool refused = false;
            try
            {
                run_dit_stage(model, prompt, 16, {}, req);
            }
            catch (const std::runtime_error &e)
            {
                refused = std::string(e.what()).find("Trace file exists") != std::string::npos;
            }
            REQUIRE(refused, "existing trace files overwritten");
            std::filesystem::remove_all(dir);

            // img2img: strength 0.5 starts at step 4 from sigma*noise + (1-sigma)*encoded
            req.trace.clear();
            req.encoded = normal(8, 6, 128, ERNIE_SYNTH_HIDDEN);
            req.strength = 0.5f;
            const DitStageResult i2i = run_dit_stage(model, prompt, 16, {}, req);
            const Img2ImgStart start = make_img2img_start(req.encoded, initial_noise(8, 6, 3), FlowSchedule::turbo(8), 0.5f);
            std::vector<DenoiseStepStats> istats;
            const Tensor i2i_hand = denoise(manual, start.latent, 8, istats, {}, start.start_step);
            REQUIRE(i2i.start_step == 4 && start.start_step == 4 && i2i.steps.size() == 4 && i2i.latent.data == i2i_hand.data,
                    "img2img DiT stage");
            req.strength = 0.f;
            const DitStageResult recon = run_dit_stage(model, prompt, 16, {}, req);
            REQUIRE(recon.start_step == 8 && recon.steps.empty() && recon.latent.data == req.encoded.data,
                    "strength 0 ran a step");
        }

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
    // the VAE stage: host and device decode agree, device RGB bytes equal rgb_image of the decoded tensor,
    // run_vae_stage equals unpack_for_vae + decode by hand and writes the reference's trace files
    try
    {
        GpuContext ctx(true, 0);
        VaeDecoder vae(ctx);
        vae.synthesize(7);
        const int w = 4, h = 3; // packed latent [128][3][4] -> image 64 x 48
        const Tensor latent = normal(w, h, 128, ERNIE_SYNTH_LATENT);
        Tensor mean(128), variance(128);
        for (int c = 0; c < 128; ++c)
        {
            mean[size_t(c)] = 0.01f * float(c % 7);
            variance[size_t(c)] = 0.5f + 0.01f * float(c % 5);
        }
        const DeviceTensor unpacked = unpack_for_vae(ctx, DeviceTensor::upload(ctx, latent), mean, variance);
        const Tensor unpacked_host = unpacked.download();
        VaeStats stats;
        const Tensor decoded = vae.decode(unpacked_host, Precision::BF16, &stats);
        REQUIRE(decoded.w == 64 && decoded.h == 48 && decoded.c == 3, "decoded shape");
        REQUIRE(stats.details.size() == 1 && stats.details[0].status == "complete", "VAE stats");
        RgbImage bytes;
        const Tensor decoded_dev = vae.decode(unpacked, Precision::BF16, &bytes).download();
        REQUIRE(decoded_dev.data == decoded.data, "host and device decode differ");
        REQUIRE(bytes.pixels == rgb_image(decoded).pixels, "device RGB bytes differ from rgb_image");
        char folder[] = "/tmp/ernie_vae_traceXXXXXX";
        REQUIRE(mkdtemp(folder) != nullptr, "trace folder");
        const VaeStageResult stage = run_vae_stage(vae, latent, mean, variance, Precision::BF16, folder);
        REQUIRE(stage.decoded.data == decoded.data && stage.image.pixels == bytes.pixels, "VAE stage differs");
        REQUIRE(stage.unpacked.data == unpacked_host.data, "VAE stage unpacked latent differs");
        for (const char *f : {"final.f32", "unpacked.f32", "decoded.f32"})
            REQUIRE(std::filesystem::file_size(std::filesystem::path(folder) / f) > 0, "missing trace " << f);
        REQUIRE(read_tensor((std::filesystem::path(folder) / "decoded.f32").string(), 64, 48, 3).data == decoded.data,
                "decoded trace");
        bool threw = false;
        try
        {
            run_vae_stage(vae, latent, mean, variance, Precision::BF16, folder); // traces exist
        }
        catch (const std::runtime_error &)
        {
            threw = true;
        }
        REQUIRE(threw, "existing trace overwritten");
        std::filesystem::remove_all(folder);
        const Tensor exact = vae.decode(unpacked_host, Precision::FP32);
        double num = 0, den = 0;
        for (size_t i = 0; i < exact.total(); ++i)
        {
            num += double(exact[i] - decoded[i]) * double(exact[i] - decoded[i]);
            den += double(exact[i]) * double(exact[i]);
        }
        REQUIRE(std::sqrt(num / den) < 0.02, "BF16 decode against FP32-exact: " << std::sqrt(num / den));
    }
    catch (const std::exception &e)
    {
        std::cerr << "VAE exception: " << e.what() << "\n";
        return 1;
    }
    // the prompt encoder: run_text_blocks with text_constants; the causal mask is required
    try
    {
        GpuContext ctx(true, 0);
        TextModel text(ctx, 2);
        text.synthesize(3);
        std::vector<float> f(64);
        for (int j = 0; j < 64; ++j) f[size_t(j)] = 1.f / std::pow(1000000.f, float(j) / 64.f);
        const int bucket = 12;
        auto k = text_constants(f, bucket);
        Tensor x = normal(3072, bucket, 1, ERNIE_SYNTH_TEXT);
        BlockSequenceStats stats;
        const Tensor y = run_text_blocks(text, x, k, Precision::BF16, stats);
        REQUIRE(y.w == 3072 && y.h == bucket && stats.compute_seconds.size() == 1, "text output shape");
        bool finite = true;
        for (size_t i = 0; i < y.total(); ++i) finite = finite && std::isfinite(y[i]);
        REQUIRE(finite, "text output finite");
        const Tensor one = run_text_blocks(text, x, k, Precision::BF16, stats, 1);
        REQUIRE(one.data != y.data, "layer count ignored");
        k[2][5] = 0.f; // a key above the diagonal unmasked
        bool threw = false;
        try
        {
            run_text_blocks(text, x, k, Precision::BF16, stats);
        }
        catch (const std::invalid_argument &)
        {
            threw = true;
        }
        REQUIRE(threw, "non-causal text mask accepted");
    }
    catch (const std::exception &e)
    {
        std::cerr << "text exception: " << e.what() << "\n";
        return 1;
    }
    // generate_from_ids: the three stages from token ids to RGB bytes, deterministic, with the traces
    try
    {
        GpuContext ctx(true, 0);
        TextModel text(ctx, 2);
        DitModel dit(ctx, 2);
        VaeDecoder vae(ctx);
        text.synthesize(3);
        dit.synthesize(11);
        vae.synthesize(7);
        char folder[] = "/tmp/ernie_generateXXXXXX";
        REQUIRE(mkdtemp(folder) != nullptr, "generate folder");
        const std::string table = std::string(folder) + "/embeddings.bf16";
        {
            std::ofstream f(table, std::ios::binary);
            for (uint32_t id : {5u, 9u, 100u})
            {
                f.seekp(std::streamoff(id) * 3072 * 2);
                for (int j = 0; j < 3072; ++j)
                {
                    const uint16_t b = ernie_synth_bf16_bits(float(0.2 * ernie_synth_normal(1, id, uint64_t(j))));
                    f.write(reinterpret_cast<const char *>(&b), 2);
                }
            }
            f.seekp(std::streamoff(131072) * 3072 * 2 - 1);
            f.put('\0'); // sparse table of the full size
        }
        std::vector<float> tf(64);
        for (int j = 0; j < 64; ++j) tf[size_t(j)] = 1.f / std::pow(1000000.f, float(j) / 64.f);
        Tensor mean(128), variance(128);
        for (int c = 0; c < 128; ++c) variance[size_t(c)] = 1.f;
        GenerationModels models{text, dit, vae, table, tf, {}, mean, variance, 8};
        DitStageRequest req;
        req.width = 64;
        req.height = 48;
        req.steps = 2;
        req.seed = 4;
        int notified = 0;
        const GeneratedImage a = generate_from_ids(models, {5, 9, 100}, 8, req,
                                                   [&](const DitStageProgress &p) { notified += p.stage == "text"; });
        const GeneratedImage b = generate_from_ids(models, {5, 9, 100}, 8, req);
        REQUIRE(a.image.width == 64 && a.image.height == 48 && a.image.pixels.size() == 64 * 48 * 3, "image shape");
        REQUIRE(a.image.pixels == b.image.pixels && a.latent.data == b.latent.data, "generate not deterministic");
        REQUIRE(notified == 1 && a.text.h == 3 && a.text.w == 3072, "text stage");
        const std::string trace = std::string(folder) + "/trace";
        std::filesystem::create_directory(trace);
        req.trace = trace;
        const GeneratedImage t = generate_from_ids(models, {5, 9, 100}, 8, req);
        for (const char *f : {"text.f32", "final.f32", "unpacked.f32", "decoded.f32"})
            REQUIRE(std::filesystem::exists(std::filesystem::path(trace) / f), "missing trace " << f);
        REQUIRE(t.image.pixels == a.image.pixels, "traced generate differs");
        // img2img (src/pipeline.cpp:341-345, :392-437, :536-540): strength 0 decodes the encoded image
        // straight back; a positive strength is generate_from_ids from the encoded latent's start step
        VaeEncoder encoder(ctx);
        encoder.synthesize(13);
        DitStageRequest ir = req;
        ir.trace.clear();
        ir.strength = 0.f;
        bool threw = false;
        try { generate_img2img_from_ids(models, {}, 8, a.image, ir); }
        catch (const std::invalid_argument &) { threw = true; }
        REQUIRE(threw, "img2img without an encoder accepted");
        models.encoder = &encoder;
        const VaeEncoding enc = encode_vae(encoder, a.image, ir.precision);
        REQUIRE(enc.mean.c == 32 && enc.mean.w == 8 && enc.mean.h == 6 && enc.normalized.c == 128 &&
                    enc.normalized.w == 4 && enc.normalized.h == 3,
                "encoding shape");
        const GeneratedImage z = generate_img2img_from_ids(models, {}, 8, a.image, ir);
        const VaeStageResult back = run_vae_stage(vae, enc.normalized, mean, variance, ir.precision);
        REQUIRE(z.image.pixels == back.image.pixels && z.latent.data == enc.normalized.data,
                "strength 0 is not encode + decode");
        ir.strength = 0.5f;
        const GeneratedImage h = generate_img2img_from_ids(models, {5, 9, 100}, 8, a.image, ir);
        DitStageRequest manual = ir;
        manual.encoded = enc.normalized;
        const GeneratedImage hm = generate_from_ids(models, {5, 9, 100}, 8, manual);
        REQUIRE(h.image.pixels == hm.image.pixels && h.start_step == hm.start_step && h.start_step > 0,
                "img2img is not the DiT stage from the encoded latent");
        const std::string itrace = std::string(folder) + "/itrace";
        std::filesystem::create_directory(itrace);
        ir.trace = itrace;
        const GeneratedImage ht = generate_img2img_from_ids(models, {5, 9, 100}, 8, a.image, ir);
        for (const char *f : {"input.rgb", "img2img.txt", "encoder-mean.f32", "encoder-packed.f32",
                              "encoder-normalized.f32", "text.f32", "final.f32"})
            REQUIRE(std::filesystem::exists(std::filesystem::path(itrace) / f), "missing img2img trace " << f);
        REQUIRE(ht.image.pixels == h.image.pixels, "traced img2img differs");
        ir.trace.clear();
        for (float bad_strength : {-0.1f, 1.5f})
        {
            ir.strength = bad_strength;
            threw = false;
            try { generate_img2img_from_ids(models, {5, 9, 100}, 8, a.image, ir); }
            catch (const std::invalid_argument &) { threw = true; }
            REQUIRE(threw, "strength " << bad_strength << " accepted");
        }
        ir.strength = 0.5f;
        RgbImage odd = a.image;
        odd.width = 40;
        odd.pixels.resize(size_t(40) * 48 * 3);
        threw = false;
        try { encode_vae(encoder, odd); }
        catch (const std::invalid_argument &) { threw = true; }
        REQUIRE(threw, "40-pixel-wide image accepted by the encoder");
        threw = false;
        try { generate_img2img_from_ids(models, {5, 9, 100}, 8, odd, ir); }
        catch (const std::invalid_argument &) { threw = true; }
        REQUIRE(threw, "img2img image of another size accepted");
        // the prompt enhancer after its tokenizer (enhance_prompt, src/prompt_enhancer.cpp:68-197): greedy and
        // seeded decoding are reproducible, every step's logits are observed, token ids stay in the vocabulary
        {
            TextModel pe(ctx, 2);
            pe.synthesize(21);
            pe.synthesize_head(21);
            PeOptions o;
            o.greedy = true;
            o.max_tokens = 6;
            int observed = 0, decode_reports = 0;
            const PeResult g1 = enhance_prompt_from_ids(
                pe, table, tf, {5, 9, 100}, o, Precision::FP32, 1,
                [&](const char *stage, int, int) { decode_reports += std::string(stage) == "decode"; },
                [&](int, const std::vector<float> &l) { observed += l.size() == 131072; });
            const PeResult g2 = enhance_prompt_from_ids(pe, table, tf, {5, 9, 100}, o, Precision::FP32, 1);
            REQUIRE(!g1.generated_ids.empty() && g1.generated_ids.size() <= 6 && g1.generated_ids == g2.generated_ids,
                    "greedy PE decode not reproducible");
            REQUIRE(observed == int(g1.generated_ids.size()) && decode_reports >= 1, "PE observers");
            for (uint32_t id : g1.generated_ids) REQUIRE(id < 131072, "PE token outside the vocabulary");
            REQUIRE(g1.eos == (g1.generated_ids.back() == 2), "PE end-of-sequence flag");
            o.greedy = false;
            o.seed = 7;
            const PeResult s1 = enhance_prompt_from_ids(pe, table, tf, {5, 9, 100}, o, Precision::BF16, 3);
            const PeResult s2 = enhance_prompt_from_ids(pe, table, tf, {5, 9, 100}, o, Precision::BF16, 3);
            REQUIRE(s1.generated_ids == s2.generated_ids, "seeded PE decode not reproducible");
            bool rejected = false;
            try { enhance_prompt_from_ids(pe, table, tf, {5}, o, Precision::BF16, 33); }
            catch (const std::invalid_argument &) { rejected = true; }
            REQUIRE(rejected, "PE prefill chunk 33 accepted");
            rejected = false;
            try { enhance_prompt_from_ids(pe, table, tf, {}, o, Precision::BF16, 1); }
            catch (const std::invalid_argument &) { rejected = true; }
            REQUIRE(rejected, "empty PE input accepted");
        }
        std::filesystem::remove_all(folder);
    }
    catch (const std::exception &e)
    {
        std::cerr << "generate exception: " << e.what() << "\n";
        return 1;
    }
    if (failures) return 1;
    std::cout << "host GPU contracts passed\n";
    return 0;
}
