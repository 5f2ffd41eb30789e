// glacier_b200.hpp -- C++17 host-side mirror of the reference's operator API
// for the MoE feed-forward hot path, over the C ABI in glacier_b200.h.
//
// Class and method names follow Glacier.Inference.Distributed so that a host
// written against the reference reads the same:
//   GpuExpertStageWorker::ProcessActivation  <- IInferenceStageWorker.ProcessActivation
//                                               (IInferenceStageWorker.cs:43,
//                                               CpuWarmExpertPoolWorker.cs:203-278)
//   GpuExpertStageWorker::ProcessRoutedTopK  <- GpuFirstExpertStageWorker.ProcessRoutedTopK
//                                               (GpuFirstExpertStageWorker.cs:416-583)
//   GpuExpertStageWorker::ForwardBatch       <- IClusterStageModel.ForwardBatchStage for a
//                                               MoE FFN layer (IClusterStageModel.cs:24)
//   QuantizationKernels                      <- Protocol/QuantizationKernels.cs:57-163
//   FusedActivationHeader                    <- Protocol/FusedActivationHeader.cs:41-218
//   ActivationHeader                         <- ActivationHeader.cs:39-57
// Errors surface as GlcException carrying the GLC_ERR_* status, the way the
// reference throws ArgumentException / ObjectDisposedException /
// NotSupportedException.  Header-only; link libglacier_b200.so.
#pragma once

#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "glacier_b200.h"

namespace glacier {
namespace b200 {

class GlcException : public std::runtime_error {
public:
    GlcException(int status, const std::string& msg) : std::runtime_error(msg), status_(status) {}
    int Status() const noexcept { return status_; }

private:
    int status_;
};

inline void Check(int status) {
    if (status != GLC_OK) throw GlcException(status, glc_last_error());
}

enum class WirePrecisionMode : uint8_t { FP32 = 0, FP16 = 1, INT8_Symmetric = 2, FP8_E4M3 = 3 };

// 32-byte stage-worker header (ActivationHeader.cs:39-57); ExpertId at offset 24.
struct ActivationHeader {
    static constexpr uint32_t ActivationMagic = 0x47414354u;
    uint32_t Magic = ActivationMagic;
    uint64_t SequenceId = 0;
    int32_t TokenIndex = 0;
    int32_t LayerIndex = 0;
    int32_t HiddenDim = 0;
    int32_t ExpertId = 0;
    uint32_t Flags = 0;
};

struct FusedActivationHeader {
    static constexpr int HeaderSize = 32;
    static constexpr uint32_t FusedMagic = 0x47414354u;
    glc_fused_header h{};

    FusedActivationHeader() = default;
    FusedActivationHeader(uint64_t seq, int32_t token, int32_t layer, int32_t dim,
                          WirePrecisionMode mode, uint8_t flags = 0, float scale = 1.0f,
                          uint16_t batch = 0) {
        h.sequence_id = seq;
        h.token_index = token;
        h.layer_index = layer;
        h.hidden_dim = dim;
        h.precision_mode = static_cast<uint8_t>(mode);
        h.flags = flags;
        h.batch_tokens = batch;
        h.scale = scale;
    }
    void WriteTo(uint8_t* destination, size_t length) const {
        if (length < HeaderSize) throw GlcException(GLC_ERR_INVALID_ARG, "Destination too small for FusedActivationHeader");
        Check(glc_fused_header_write(&h, destination));
    }
    static FusedActivationHeader ReadFrom(const uint8_t* source, size_t length) {
        if (length < HeaderSize) throw GlcException(GLC_ERR_INVALID_ARG, "Source too small for FusedActivationHeader");
        FusedActivationHeader r;
        Check(glc_fused_header_read(source, &r.h));
        return r;
    }
    int GetPayloadByteCount() const { return glc_fused_header_payload_bytes(&h); }
};

struct QuantizationKernels {
    static int GetPackedTokenBytes(WirePrecisionMode mode, int dim) {
        return glc_wire_token_bytes(static_cast<int32_t>(mode), dim);
    }
    static int GetPackedBatchBytes(WirePrecisionMode mode, int dim, int tokenCount) {
        return GetPackedTokenBytes(mode, dim) * tokenCount;
    }
    static void QuantizeBatch(const float* input, size_t inputLength, uint8_t* destination,
                              size_t destinationLength, int dim, int tokenCount, WirePrecisionMode mode) {
        if (inputLength < (size_t)dim * (size_t)tokenCount)
            throw GlcException(GLC_ERR_INVALID_ARG, "Input float span smaller than dim * tokenCount");
        Check(glc_wire_quantize(static_cast<int32_t>(mode), input, tokenCount, dim, destination, destinationLength));
    }
    static void DequantizeBatch(const uint8_t* source, size_t sourceLength, float* destination,
                                size_t destinationLength, int dim, int tokenCount, WirePrecisionMode mode) {
        if (destinationLength < (size_t)dim * (size_t)tokenCount)
            throw GlcException(GLC_ERR_INVALID_ARG, "Destination float span smaller than dim * tokenCount");
        Check(glc_wire_dequantize(static_cast<int32_t>(mode), source, sourceLength, tokenCount, dim, destination));
    }
    // Returns the scale written to bytes 0..3 (1.0 for unscaled formats).
    static float QuantizeToken(const float* input, int dim, uint8_t* destination, size_t destinationLength,
                               WirePrecisionMode mode) {
        QuantizeBatch(input, (size_t)dim, destination, destinationLength, dim, 1, mode);
        float scale = 1.0f;
        if (mode == WirePrecisionMode::INT8_Symmetric || mode == WirePrecisionMode::FP8_E4M3)
            std::memcpy(&scale, destination, 4);
        return scale;
    }
    static void DequantizeToken(const uint8_t* source, size_t sourceLength, float* destination, int dim,
                                WirePrecisionMode mode) {
        DequantizeBatch(source, sourceLength, destination, (size_t)dim, dim, 1, mode);
    }
};

// The slot counters of GpuFirstExpertStageWorker.GetTelemetry
// (GpuFirstExpertStageWorker.cs:763-783).
struct GpuFirstWorkerTelemetry {
    int64_t GpuResidentSlotCapacity = 0;
    int64_t GpuVramHitCount = 0;
    int64_t GpuPcieTransferCount = 0;
    int64_t LookaheadPrefetchCount = 0;
};

// One MoE layer family resident in one GPU's HBM (GGUF Q4_K experts).
class GpuExpertStageWorker {
public:
    explicit GpuExpertStageWorker(const glc_moe_desc& desc) : desc_(desc) { Check(glc_moe_create(&desc_, &h_)); }
    ~GpuExpertStageWorker() { Dispose(); }
    GpuExpertStageWorker(const GpuExpertStageWorker&) = delete;
    GpuExpertStageWorker& operator=(const GpuExpertStageWorker&) = delete;
    GpuExpertStageWorker(GpuExpertStageWorker&& o) noexcept : desc_(o.desc_), h_(std::exchange(o.h_, nullptr)) {}

    int HiddenDim() const { return desc_.hidden_dim; }
    int ExpertFfnDim() const { return desc_.expert_ffn_dim; }
    int NumExperts() const { return desc_.num_experts; }

    void Dispose() {
        if (h_) {
            glc_moe_destroy(h_);
            h_ = nullptr;
        }
    }
    void LoadLayer(int layer, const glc_layer_weights& w) { Check(glc_moe_load_layer(Handle(), layer, &w)); }
    void SynthLayer(int layer, uint64_t seed) { Check(glc_moe_synth_layer(Handle(), layer, seed)); }

    // Expert residency (before the first LoadLayer / SynthLayer): the routed
    // experts in pinned host memory and `gpuSlotCapacity` of them in HBM slots.
    void SetExpertSlots(int gpuSlotCapacity) { Check(glc_moe_set_expert_slots(Handle(), gpuSlotCapacity)); }
    // Router lookahead prefetch (GpuFirstExpertStageWorker.cs:388-407).
    void PrefetchLookaheadExperts(int nextLayerIdx, const int32_t* predictedExpertIds, int count) {
        Check(glc_moe_prefetch_experts(Handle(), nextLayerIdx, predictedExpertIds, count));
    }
    GpuFirstWorkerTelemetry GetTelemetry() {
        int64_t v[4] = {};
        Check(glc_moe_expert_residency(Handle(), v));
        GpuFirstWorkerTelemetry t;
        t.GpuResidentSlotCapacity = v[0];
        t.GpuVramHitCount = v[1];
        t.GpuPcieTransferCount = v[2];
        t.LookaheadPrefetchCount = v[3];
        return t;
    }

    // Allocating form: the output buffer belongs to the caller (the reference
    // returns a RefCountedPartitionBuffer the caller disposes).
    std::vector<float> ProcessActivation(const ActivationHeader& header, const float* input, size_t inputLength) {
        std::vector<float> out((size_t)desc_.hidden_dim);
        ProcessActivation(header, input, inputLength, out.data());
        return out;
    }
    // Zero-allocation form (CpuWarmExpertPoolWorker.cs:232).
    void ProcessActivation(const ActivationHeader& header, const float* input, size_t inputLength, float* output) {
        if (inputLength < (size_t)desc_.hidden_dim)
            throw GlcException(GLC_ERR_INVALID_ARG, "Input activation is smaller than the hidden dimension");
        Check(glc_expert_forward(Handle(), header.LayerIndex, header.ExpertId, input, output));
    }
    void ProcessRoutedTopK(int layerIdx, const float* inputX, const int32_t* selectedExpertIds,
                           const float* selectedWeights, int topK, float* outputX) {
        Check(glc_routed_topk(Handle(), layerIdx, inputX, selectedExpertIds, selectedWeights, topK, outputX));
    }
    // Router + dispatch + experts + combine for T tokens (T == 1: decode GEMVs,
    // T > 1: grouped tensor-core GEMMs).
    void ForwardBatch(int layer, const float* inputXBatch, int tokens, uint32_t flags, float* outputXBatch,
                      int32_t* expertIds = nullptr, float* expertWeights = nullptr) {
        Check(glc_moe_forward(Handle(), layer, inputXBatch, tokens, flags, outputXBatch, expertIds, expertWeights));
    }

private:
    glc_moe* Handle() const {
        if (!h_) throw GlcException(GLC_ERR_DISPOSED, "GpuExpertStageWorker was disposed");
        return h_;
    }
    glc_moe_desc desc_;
    glc_moe* h_ = nullptr;
};

}  // namespace b200
}  // namespace glacier
