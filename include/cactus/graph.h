// CactusGraph — the reference's op-graph API (cactus/graph/graph.h:99-500) backed by the
// B200 kernels of include/cactus_b200.h.
//
// Same class and method names, argument meaning and error behaviour (std::runtime_error /
// std::invalid_argument) as the reference for the hot-path ops. Differences, all forced by
// buffers living in HBM:
//  * tensors are device buffers; set_input copies host data in, get_output copies the node's
//    result to a host mirror and returns it (valid until the next execute / reset);
//  * set_external_input and set_grouped_scales accept host or device pointers (host data is
//    copied to the device once);
//  * `__fp16` does not exist on x86: fp16 data is passed as 16-bit IEEE binary16 words;
//  * an INT8 right-hand side without group scales is rejected (the reference would
//    reinterpret it as fp16, graph_ops_nn.cpp:211-229).
// Ops outside the quantized transformer path (conv, bilinear, reductions, topk, ...) are not
// provided by this backend.
#pragma once
#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

#ifndef CACTUS_GRAPH_API
#define CACTUS_GRAPH_API __attribute__((visibility("default")))
#endif

enum class Precision { INT8, FP16, FP32, INT4 };
enum class ComputeBackend { CPU, NPU };

enum class OpType {
    INPUT, PRECISION_CAST,
    ADD, ADD_CLIPPED, SUBTRACT, MULTIPLY, DIVIDE,
    MATMUL, TRANSPOSE, RESHAPE, SLICE, GATHER, EMBEDDING,
    BILINEAR_INTERPOLATION,
    SUM, MEAN, VARIANCE, MIN, MAX,
    RMS_NORM, ROPE, SOFTMAX, ATTENTION, ATTENTION_INT8_HYBRID, CONV1D_CAUSAL, CONV1D_K3,
    SCALAR_ADD, SCALAR_SUBTRACT, SCALAR_MULTIPLY, SCALAR_DIVIDE, SCALAR_EXP, SCALAR_SQRT, SCALAR_COS, SCALAR_SIN,
    SILU, GELU, GELU_ERF,
    SAMPLE, CONCAT,
    SCATTER_TOPK,
    TOPK, LAYERNORM,
    INDEX,
    QUANTIZE_ACTIVATIONS,
};

struct PrecisionTraits {
    static constexpr size_t size_of(Precision p) {
        return p == Precision::FP16 ? 2 : p == Precision::FP32 ? 4 : 1;
    }
    static constexpr size_t packed_size_of(Precision p, size_t count) {
        return p == Precision::INT4 ? (count + 1) / 2 : count * size_of(p);
    }
};

struct CACTUS_GRAPH_API BufferDesc {
    std::vector<size_t> shape;
    size_t total_size = 0;
    size_t byte_size = 0;
    Precision precision = Precision::INT8;
    void* device_data = nullptr;        // HBM
    bool owns_data = false;
    std::vector<uint8_t> host_mirror;   // filled by get_output
    size_t group_size = 0, num_groups = 0;
    void* scales_data = nullptr;        // device fp16 [rows, num_groups]
    bool owns_scales = false;
    bool packed_int4 = false;
    float* activation_scales = nullptr; // device fp32 [rows] (QUANTIZE_ACTIVATIONS output)
    size_t num_rows_for_activation_scales = 0;

    BufferDesc() = default;
    BufferDesc(const std::vector<size_t>& s, Precision p);
    bool is_grouped_int8() const { return precision == Precision::INT8 && group_size > 0; }
    bool is_packed_int4() const { return packed_int4; }
    bool has_activation_scales() const { return activation_scales && num_rows_for_activation_scales > 0; }
};

struct OpParams {
    float scalar = 0.0f;
    float scale = 1.0f;
    float theta = 10000.0f;
    float epsilon = 1e-6f;
    int axis = -1;
    bool pretransposed_rhs = false;
    size_t position_offset = 0;
    size_t window_size = 0;
    bool is_causal = true;
    std::vector<size_t> new_shape;
    Precision output_precision = Precision::INT8;
    ComputeBackend backend = ComputeBackend::CPU;
    float temperature = 1.0f;
    float top_p = 1.0f;
    size_t top_k = 0;
    size_t random_seed = 0;
    size_t index_value = 0;
    const int8_t* cached_keys_int8 = nullptr;
    const int8_t* cached_values_int8 = nullptr;
    const float* cached_k_scales = nullptr;
    const float* cached_v_scales = nullptr;
    size_t cache_seq_len = 0;
    size_t num_kv_heads = 0;
    size_t head_dim = 0;
    size_t dilation = 1;  // CONV1D_CAUSAL
    size_t stride = 1;    // CONV1D_K3
};

struct GraphNode {
    size_t id;
    OpType op_type;
    std::vector<size_t> input_ids;
    BufferDesc output_buffer;
    OpParams params;
    GraphNode(size_t node_id, OpType type) : id(node_id), op_type(type) {}
};

class CACTUS_GRAPH_API CactusGraph {
public:
    CactusGraph();
    ~CactusGraph();
    CactusGraph(const CactusGraph&) = delete;
    CactusGraph& operator=(const CactusGraph&) = delete;

    size_t input(const std::vector<size_t>& shape, Precision precision = Precision::INT8);
    size_t quantize_activations(size_t input);

    size_t add(size_t input1, size_t input2);
    size_t add_clipped(size_t input1, size_t input2);
    size_t multiply(size_t input1, size_t input2);
    size_t scalar_multiply(size_t input, float value);
    size_t silu(size_t input);
    size_t gelu(size_t input);

    size_t matmul(size_t input1, size_t input2, bool pretransposed_rhs = false,
                  ComputeBackend backend = ComputeBackend::CPU);
    size_t transpose(size_t input, ComputeBackend backend = ComputeBackend::CPU);
    size_t reshape(size_t input, const std::vector<size_t>& new_shape);
    size_t index(size_t input, size_t index_value, int dim);

    size_t mmap_embeddings(const std::string& filename);
    size_t mmap_weights(const std::string& filename);
    void set_grouped_scales(size_t node_id, size_t group_size, size_t num_groups, void* scales_ptr);
    size_t embedding(const std::string& filename, size_t indices);
    size_t embedding(size_t embedding_tensor, size_t indices);

    size_t rms_norm(size_t input, size_t weight, float epsilon = 1e-5f);
    // fp16 input [rows, features], fp16 weight and bias [features] (graph_ops_nn.cpp:373-457)
    size_t layernorm(size_t input, size_t weight, size_t bias, float epsilon = 1e-5f);
    // depthwise causal conv: fp16 input [N, L, C], fp16 weight [C, 1, K] (graph_ops_nn.cpp:459-530)
    size_t conv1d_causal(size_t input, size_t weight, size_t kernel_size, size_t dilation = 1);
    // kernel-3 conv, padding 1: fp16 input [N, C_in, L], fp16 weight [C_out, C_in, 3] (graph_ops_nn.cpp:532-580)
    size_t conv1d_k3(size_t input, size_t weight, size_t stride);
    size_t rope(size_t input, float theta, size_t position_offset = 0, ComputeBackend backend = ComputeBackend::CPU);
    size_t softmax(size_t input, int axis = -1);
    size_t attention(size_t query, size_t key, size_t value, float scale, bool is_causal = true,
                     ComputeBackend backend = ComputeBackend::CPU);
    size_t attention(size_t query, size_t key, size_t value, float scale, size_t position_offset,
                     ComputeBackend backend = ComputeBackend::CPU);
    size_t attention(size_t query, size_t key, size_t value, float scale, size_t position_offset, size_t window_size,
                     ComputeBackend backend = ComputeBackend::CPU);
    size_t attention_int8_hybrid(size_t query, size_t key_new, size_t value_new, float scale, size_t position_offset,
                                 const int8_t* cached_keys, const int8_t* cached_values, const float* k_scales,
                                 const float* v_scales, size_t cache_len, size_t num_kv_heads, size_t head_dim);
    // logit_bias is accepted for API parity and has no effect: the reference adds it to a copy
    // of the logits that its temperature step then overwrites (kernel_nn.cpp:473-494)
    size_t sample(size_t logits, float temperature = 0.6f, float top_p = 0.95f, size_t top_k = 20,
                  const std::unordered_map<uint32_t, float>& logit_bias = {});

    void set_input(size_t node_id, const void* data, Precision precision);
    void set_external_input(size_t node_id, void* data, Precision precision);
    void* get_output(size_t node_id);

    void execute(const std::string& profile_file = "");
    void hard_reset();
    void soft_reset();

    size_t add_node(OpType op_type, const std::vector<size_t>& inputs, const std::vector<size_t>& output_shape,
                    const OpParams& params = {});
    const BufferDesc& get_output_buffer(size_t node_id) const;
    size_t get_node_count() const { return nodes_.size(); }

    std::vector<std::unique_ptr<GraphNode>> nodes_;
    std::unordered_map<size_t, size_t> node_index_map_;

private:
    void compute_node(GraphNode& node);
    void* ensure_device(BufferDesc& b);
    void* scratch(size_t bytes);
    size_t next_node_id_ = 0;
    std::unordered_map<std::string, size_t> weight_cache_;
    void* stream_ = nullptr;
    std::vector<void*> scratch_;
    std::vector<size_t> scratch_bytes_;
    size_t scratch_used_ = 0;
    std::vector<uint32_t> sample_history_;
};
