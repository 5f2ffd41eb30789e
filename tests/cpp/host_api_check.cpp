// Exercises the C++ host mirror (include/glacier_b200.hpp) through the C ABI.
// "cpu" mode checks the host-only entry points (header layout, sizes, errors);
// "gpu" mode also runs one expert of a synthetic layer and a routed top-k step.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <vector>

#include "glacier_b200.hpp"

using namespace glacier::b200;

static int fails = 0;
#define EXPECT(c)                                                        \
    do {                                                                 \
        if (!(c)) { std::printf("FAILED: %s (line %d)\n", #c, __LINE__); ++fails; } \
    } while (0)

int main(int argc, char** argv) {
    const bool gpu = argc > 1 && std::strcmp(argv[1], "gpu") == 0;
    // FusedActivationHeader round trip (DynamicMultiPrecisionWireTests.cs:35-60).
    FusedActivationHeader h(0x1234567890ABCDEFull, 42, 17, 5120, WirePrecisionMode::INT8_Symmetric, 6, 0.0357f, 64);
    uint8_t buf[32];
    h.WriteTo(buf, sizeof(buf));
    EXPECT(buf[0] == 0x54 && buf[1] == 0x43 && buf[2] == 0x41 && buf[3] == 0x47);
    FusedActivationHeader r = FusedActivationHeader::ReadFrom(buf, sizeof(buf));
    EXPECT(r.h.sequence_id == 0x1234567890ABCDEFull && r.h.batch_tokens == 64 && r.h.scale == 0.0357f);
    EXPECT(r.GetPayloadByteCount() == 5124 * 64);
    EXPECT(QuantizationKernels::GetPackedTokenBytes(WirePrecisionMode::INT8_Symmetric, 5120) == 5124);
    buf[0] ^= 0xFF;
    bool threw = false;
    try { FusedActivationHeader::ReadFrom(buf, sizeof(buf)); } catch (const GlcException& e) { threw = e.Status() == GLC_ERR_INVALID_ARG; }
    EXPECT(threw);
    if (gpu) {
        glc_moe_desc d{};
        d.hidden_dim = 512; d.expert_ffn_dim = 1024; d.num_experts = 4; d.top_k = 2; d.renormalize = 1;
        d.weight_type = GLC_GGUF_Q4_K; d.device = 0; d.num_layers = 1; d.max_tokens = 4;
        GpuExpertStageWorker w(d);
        w.SynthLayer(0, 99);
        std::vector<float> x(512);
        for (int i = 0; i < 512; ++i) x[i] = std::sin(0.01f * i);
        ActivationHeader ah;
        ah.ExpertId = 2;
        std::vector<float> y = w.ProcessActivation(ah, x.data(), x.size());
        double n = 0;
        for (float v : y) n += (double)v * v;
        EXPECT(std::isfinite(n) && n > 0);
        const int32_t ids[2] = {2, 2};
        const float wts[2] = {0.5f, 0.5f};
        std::vector<float> o(512);
        w.ProcessRoutedTopK(0, x.data(), ids, wts, 2, o.data());
        double diff = 0, ref = 0;
        for (int i = 0; i < 512; ++i) { diff += std::fabs(o[i] - y[i]); ref += std::fabs(y[i]); }
        EXPECT(diff <= 1e-5 * ref);
        // the same layer with two HBM slots: experts 0 and 1 are staged when
        // it is made; expert 2 is paged in on first use, then hit
        GpuExpertStageWorker pw(d);
        pw.SetExpertSlots(2);
        pw.SynthLayer(0, 99);
        std::vector<float> py = pw.ProcessActivation(ah, x.data(), x.size());
        EXPECT(std::memcmp(py.data(), y.data(), sizeof(float) * 512) == 0);
        std::vector<float> po(512);
        pw.ProcessRoutedTopK(0, x.data(), ids, wts, 2, po.data());
        EXPECT(std::memcmp(po.data(), o.data(), sizeof(float) * 512) == 0);
        const int32_t next[1] = {3};
        pw.PrefetchLookaheadExperts(0, next, 1);
        const GpuFirstWorkerTelemetry t = pw.GetTelemetry();
        EXPECT(t.GpuResidentSlotCapacity == 2 && t.GpuPcieTransferCount == 1 && t.GpuVramHitCount == 2 &&
               t.LookaheadPrefetchCount == 1);
        EXPECT(w.GetTelemetry().GpuResidentSlotCapacity == 4);  // every expert resident
        w.Dispose();
        threw = false;
        try { w.ProcessActivation(ah, x.data(), x.size()); } catch (const GlcException& e) { threw = e.Status() == GLC_ERR_DISPOSED; }
        EXPECT(threw);
    }
    std::printf("%s host API checks: %s\n", gpu ? "gpu" : "cpu", fails ? "FAILED" : "ok");
    return fails ? 1 : 0;
}
