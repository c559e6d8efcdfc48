// A small ncnn-style graph runtime for the ncnn-surface layers: it reads an
// ncnn .param (text) / .bin pair, instantiates the registered custom layers
// (SeedVR2's AdaptiveWindowAttention and SharedLinear, through their
// creators, as seedvr2_dit.cpp:614-618 registers them with ncnn::Net) plus
// the few built-in layers a DiT block graph places between them, and runs
// named-blob extraction (seedvr2_dit.cpp:730-738, :832-833) with every blob
// resident on the GPU.  ncnn itself is not part of this build; with
// S2_WITH_NCNN the same layer classes register with ncnn::Net instead.
//
// Built-in layers: Input, Split, MemoryData, BinaryOp (op_type 0 add, 1 sub,
// 2 mul, 3 div; a [1][w] operand broadcast over rows; with_scalar), RMSNorm
// and LayerNorm (ncnn param ids 0 affine_size, 1 eps, 2 affine), GELU (0
// fast_gelu), on fp32 [h][w] device blobs through libseedvr2_cuda.  Custom
// layers of this library run their device forward (forward_cuda); any other
// registered custom layer runs its host forward(Mat) (download / upload).
//
// Formats (ncnn's): .param = magic 7767517, "layer_count blob_count", then
// one line per layer "type name bottoms tops bottom... top... id=value...";
// array parameters (id <= -23300) are read and ignored.  .bin = each layer's
// load_model reads in turn: ModelBin::load(w, 1) w raw fp32 values,
// load(w, 0) a 4-byte tag then w values (tag 0 raw fp32, 0x01306B47 fp16
// padded to 4 bytes).
#pragma once

#include <map>
#include <memory>
#include <string>
#include <vector>

#include "adaptive_window_attention.h"

namespace seedvr2 {

typedef ncnn::Layer* (*layer_creator_func)(void* userdata);
typedef void (*layer_destroyer_func)(ncnn::Layer* layer, void* userdata);

class Extractor;

class Net
{
public:
    Net();
    ~Net();
    // ncnn::Net::register_custom_layer: creators are looked up by type name
    // when the .param is loaded, so register before load_param.
    int register_custom_layer(const char* type, layer_creator_func creator, layer_destroyer_func destroyer = 0,
                              void* userdata = 0);
    int load_param(const char* path);
    int load_param_mem(const char* text);
    int load_model(const char* path);
    int load_model_mem(const unsigned char* data, size_t size);
    Extractor create_extractor() const;
    void clear();

    int blob_index(const char* name) const;
    int layer_count() const { return static_cast<int>(layers.size()); }
    int blob_count() const { return static_cast<int>(blob_names.size()); }

private:
    friend class Extractor;
    struct Custom
    {
        std::string type;
        layer_creator_func creator;
        layer_destroyer_func destroyer;
        void* userdata;
    };
    struct Entry
    {
        std::string type, name;
        std::vector<int> bottoms, tops;
        ncnn::ParamDict pd;
        ncnn::Layer* layer = nullptr; // custom layers
        int custom = -1;
        // built-ins
        int op = 0, with_scalar = 0, affine = 0, affine_size = 0, fast = 0;
        float scalar = 0.f, eps = 0.f;
        int w = 0, h = 0, c = 0;
        ncnn::Mat data, gamma, beta;
        mutable float* d_data = nullptr; // device copies (MemoryData data; gamma then beta)
        mutable float* d_gamma = nullptr;
        mutable float* d_beta = nullptr;
    };
    int parse_param(const std::string& text);
    int load_weights(const ncnn::ModelBin& mb);
    int upload(const Entry& e) const;

    // device memory of the blobs: a caching pool (ncnn's PoolAllocator
    // role) so repeated extractions allocate nothing once warm
    std::shared_ptr<void> blob_alloc(size_t bytes) const;
    struct Pool;
    std::shared_ptr<Pool> pool;

    std::vector<Custom> customs;
    std::vector<Entry> layers;
    std::vector<std::string> blob_names;
    std::vector<int> blob_producer;  // layer index
    std::vector<int> blob_consumers; // number of consuming layers
    bool model_loaded = false;
};

// One extraction session (ncnn::Extractor): inputs are bound by name, blobs
// are computed on demand, intermediate device blobs are released once every
// consumer has run (ncnn's light mode) and recomputed if asked for again.
class Extractor
{
public:
    ~Extractor();
    Extractor(Extractor&& other);
    // host fp32 [h][w] Mat (dims 2; a 1-D Mat is one row)
    int input(const char* blob_name, const ncnn::Mat& in);
    // device fp32 blob, borrowed (must stay valid until extraction is done)
    int input_cuda(const char* blob_name, const CudaBlob& in);
    int extract(const char* blob_name, ncnn::Mat& out);
    // device fp32 blob owned by this extractor (valid until it is destroyed)
    int extract_cuda(const char* blob_name, CudaBlob& out);

private:
    friend class Net;
    explicit Extractor(const Net* net);
    Extractor(const Extractor&) = delete;
    struct Slot
    {
        CudaBlob b;
        bool owned = false;
        bool input = false;
        bool pinned = false; // handed out by extract_cuda: never released
        int pending = 0;     // consumers that have not run yet
    };
    int compute(int blob, int depth);
    int run_layer(int li, int depth);
    int alloc(Slot& s, int w, int h);
    void release(int blob);
    const Net* net;
    std::vector<Slot> slots;
    std::vector<std::shared_ptr<void> > mem; // device memory per blob (Split tops share their bottom's)
};

} // namespace seedvr2
