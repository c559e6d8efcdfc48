// The ncnn-style graph runtime of the ncnn-surface layers (see net.h).
#include "net.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <sstream>

#include "shared_linear.h"

namespace seedvr2 {

namespace {

constexpr int kParamMagic = 7767517;
constexpr uint32_t kTagFp16 = 0x01306B47u;

bool is_float_token(const std::string& s)
{
    return s.find_first_of(".eE") != std::string::npos &&
           !(s.size() > 1 && (s[0] == '0') && (s[1] == 'x' || s[1] == 'X'));
}

float half_to_float(uint16_t h)
{
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
    if (exp == 0)
    {
        if (man == 0)
            bits = sign;
        else
        {
            // subnormal half: normalise into a float
            exp = 127 - 15 + 1;
            while (!(man & 0x400u))
            {
                man <<= 1;
                exp--;
            }
            bits = sign | (exp << 23) | ((man & 0x3FFu) << 13);
        }
    }
    else if (exp == 31)
        bits = sign | 0x7F800000u | (man << 13);
    else
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// ModelBin over the bytes of a .bin (ncnn's ModelBinFromDataReader).
class ByteModelBin : public ncnn::ModelBin
{
public:
    ByteModelBin(const unsigned char* d, size_t n) : data(d), size(n) {}
    virtual ncnn::Mat load(int w, int type) const
    {
        if (w <= 0) return ncnn::Mat();
        uint32_t tag = 0;
        if (type == 0)
        {
            if (!take(&tag, 4)) return ncnn::Mat();
            if (tag != 0 && tag != kTagFp16) return ncnn::Mat(); // quantised forms are not supported
        }
        else if (type != 1)
            return ncnn::Mat();
        ncnn::Mat m(w);
        if (m.empty()) return m;
        if (tag == kTagFp16)
        {
            std::vector<uint16_t> h((size_t)w);
            if (!take(h.data(), (size_t)w * 2)) return ncnn::Mat();
            if (((size_t)w * 2) % 4) cursor += 2; // ncnn pads fp16 arrays to 4 bytes
            for (int i = 0; i < w; i++) ((float*)m.data)[i] = half_to_float(h[i]);
            return m;
        }
        if (!take(m.data, (size_t)w * 4)) return ncnn::Mat();
        return m;
    }
    bool exhausted() const { return cursor == size; }

private:
    bool take(void* dst, size_t n) const
    {
        if (cursor + n > size) return false;
        std::memcpy(dst, data + cursor, n);
        cursor += n;
        return true;
    }
    const unsigned char* data;
    size_t size;
    mutable size_t cursor = 0;
};

bool read_file(const char* path, std::vector<unsigned char>& out)
{
    FILE* f = std::fopen(path, "rb");
    if (!f) return false;
    std::fseek(f, 0, SEEK_END);
    const long n = std::ftell(f);
    std::fseek(f, 0, SEEK_SET);
    out.resize(n > 0 ? (size_t)n : 0);
    const bool ok = n >= 0 && std::fread(out.data(), 1, out.size(), f) == out.size();
    std::fclose(f);
    return ok;
}

} // namespace

// ---------------------------------------------------------------- Net
// Freed blocks are kept by size and handed out again for requests of up to
// their size (and at least half of it); everything is released with the Net.
struct Net::Pool
{
    std::mutex m;
    std::multimap<size_t, void*> free_blocks;
    ~Pool()
    {
        for (auto& kv : free_blocks) cudaFree(kv.second);
    }
};

std::shared_ptr<void> Net::blob_alloc(size_t bytes) const
{
    bytes = (bytes + 255) & ~size_t(255);
    std::shared_ptr<Pool> p = pool;
    void* ptr = nullptr;
    {
        std::lock_guard<std::mutex> lock(p->m);
        auto it = p->free_blocks.lower_bound(bytes);
        if (it != p->free_blocks.end() && it->first <= 2 * bytes)
        {
            ptr = it->second;
            bytes = it->first;
            p->free_blocks.erase(it);
        }
    }
    if (!ptr && cudaMalloc(&ptr, bytes ? bytes : 256) != cudaSuccess) return nullptr;
    return std::shared_ptr<void>(ptr, [p, bytes](void* q) {
        std::lock_guard<std::mutex> lock(p->m);
        p->free_blocks.emplace(bytes, q);
    });
}

Net::Net() : pool(std::make_shared<Pool>()) {}

Net::~Net()
{
    clear();
}

void Net::clear()
{
    for (Entry& e : layers)
    {
        if (e.layer)
        {
            const Custom& c = customs[e.custom];
            if (c.destroyer)
                c.destroyer(e.layer, c.userdata);
            else
                delete e.layer;
        }
        if (e.d_data) cudaFree(e.d_data);
        if (e.d_gamma) cudaFree(e.d_gamma);
        if (e.d_beta) cudaFree(e.d_beta);
    }
    layers.clear();
    blob_names.clear();
    blob_producer.clear();
    blob_consumers.clear();
    model_loaded = false;
}

int Net::register_custom_layer(const char* type, layer_creator_func creator, layer_destroyer_func destroyer,
                               void* userdata)
{
    if (!type || !creator) return -1;
    for (Custom& c : customs)
        if (c.type == type)
        {
            c.creator = creator;
            c.destroyer = destroyer;
            c.userdata = userdata;
            return 0;
        }
    customs.push_back({type, creator, destroyer, userdata});
    return 0;
}

int Net::blob_index(const char* name) const
{
    if (!name) return -1;
    for (size_t i = 0; i < blob_names.size(); i++)
        if (blob_names[i] == name) return static_cast<int>(i);
    return -1;
}

int Net::load_param(const char* path)
{
    std::vector<unsigned char> bytes;
    if (!path || !read_file(path, bytes)) return -1;
    return parse_param(std::string(bytes.begin(), bytes.end()));
}

int Net::load_param_mem(const char* text)
{
    if (!text) return -1;
    return parse_param(text);
}

int Net::parse_param(const std::string& text)
{
    clear();
    std::istringstream in(text);
    std::string line;
    int magic = 0, layer_count = 0, blob_count = 0;
    if (!(in >> magic) || magic != kParamMagic || !(in >> layer_count >> blob_count) || layer_count <= 0 ||
        blob_count <= 0)
        return -1;
    std::getline(in, line);
    std::map<std::string, int> blob_of;
    for (int li = 0; li < layer_count; li++)
    {
        do
        {
            if (!std::getline(in, line)) return -1;
        } while (line.find_first_not_of(" \t\r") == std::string::npos);
        std::istringstream ls(line);
        Entry e;
        int nb = 0, nt = 0;
        if (!(ls >> e.type >> e.name >> nb >> nt) || nb < 0 || nt < 0) return -1;
        for (int i = 0; i < nb; i++)
        {
            std::string b;
            if (!(ls >> b)) return -1;
            auto it = blob_of.find(b);
            if (it == blob_of.end()) return -1; // consumed before produced
            e.bottoms.push_back(it->second);
            blob_consumers[it->second]++;
        }
        for (int i = 0; i < nt; i++)
        {
            std::string t;
            if (!(ls >> t) || blob_of.count(t)) return -1;
            const int idx = static_cast<int>(blob_names.size());
            blob_of[t] = idx;
            blob_names.push_back(t);
            blob_producer.push_back(li);
            blob_consumers.push_back(0);
            e.tops.push_back(idx);
        }
        std::string kv;
        while (ls >> kv)
        {
            const size_t eq = kv.find('=');
            if (eq == std::string::npos) return -1;
            const int id = std::atoi(kv.substr(0, eq).c_str());
            if (id <= -23300) continue; // array parameter: not used by these layers
            const std::string v = kv.substr(eq + 1);
            if (is_float_token(v))
                e.pd.set(id, (float)std::atof(v.c_str()));
            else
                e.pd.set(id, std::atoi(v.c_str()));
        }
        int custom = -1;
        for (size_t c = 0; c < customs.size(); c++)
            if (customs[c].type == e.type) custom = static_cast<int>(c);
        if (custom >= 0)
        {
            e.custom = custom;
            e.layer = customs[custom].creator(customs[custom].userdata);
            layers.push_back(e); // owns e.layer from here (clear() frees it)
            if (!layers.back().layer || layers.back().layer->load_param(layers.back().pd) != 0) return -1;
            continue;
        }
        if (e.type == "Input" || e.type == "Split")
        {
            if ((e.type == "Input" && (nb != 0 || nt != 1)) || (e.type == "Split" && nb != 1)) return -1;
        }
        else if (e.type == "MemoryData")
        {
            e.w = e.pd.get(0, 0);
            e.h = e.pd.get(1, 0);
            e.c = e.pd.get(2, 0);
            if (e.w <= 0 || e.h < 0 || e.c < 0 || nb != 0 || nt != 1) return -1;
        }
        else if (e.type == "BinaryOp")
        {
            e.op = e.pd.get(0, 0);
            e.with_scalar = e.pd.get(1, 0);
            e.scalar = e.pd.get(2, 0.f);
            if (e.op < 0 || e.op > 3 || nt != 1 || nb != (e.with_scalar ? 1 : 2)) return -1;
        }
        else if (e.type == "RMSNorm" || e.type == "LayerNorm")
        {
            e.affine_size = e.pd.get(0, 0);
            e.eps = e.pd.get(1, 0.001f);
            e.affine = e.pd.get(2, 1);
            if (nb != 1 || nt != 1 || (e.affine && e.affine_size <= 0)) return -1;
        }
        else if (e.type == "GELU")
        {
            e.fast = e.pd.get(0, 0);
            if (nb != 1 || nt != 1) return -1;
        }
        else
        {
            std::fprintf(stderr, "seedvr2::Net: layer %s not exists or registered\n", e.type.c_str());
            return -1;
        }
        layers.push_back(e);
    }
    return static_cast<int>(blob_names.size()) == blob_count ? 0 : -1;
}

int Net::load_model(const char* path)
{
    std::vector<unsigned char> bytes;
    if (!path || !read_file(path, bytes)) return -1;
    return load_model_mem(bytes.data(), bytes.size());
}

int Net::load_model_mem(const unsigned char* data, size_t size)
{
    if (layers.empty()) return -1;
    ByteModelBin mb(data, size);
    const int r = load_weights(mb);
    if (r != 0) return r;
    model_loaded = true;
    return 0;
}

int Net::load_weights(const ncnn::ModelBin& mb)
{
    for (Entry& e : layers)
    {
        if (e.layer)
        {
            const int r = e.layer->load_model(mb);
            if (r != 0) return r;
        }
        else if (e.type == "MemoryData")
        {
            e.data = mb.load(e.w * (e.h > 0 ? e.h : 1) * (e.c > 0 ? e.c : 1), 1);
            if (e.data.empty()) return -100;
        }
        else if ((e.type == "RMSNorm" || e.type == "LayerNorm") && e.affine)
        {
            e.gamma = mb.load(e.affine_size, 1);
            if (e.gamma.empty()) return -100;
            if (e.type == "LayerNorm")
            {
                e.beta = mb.load(e.affine_size, 1);
                if (e.beta.empty()) return -100;
            }
        }
    }
    return 0;
}

// Device copies of a built-in layer's weights, made on first use.
int Net::upload(const Entry& e) const
{
    auto put = [](const ncnn::Mat& m, float*& dst) {
        if (dst || m.empty()) return 0;
        const size_t n = (size_t)m.w * (m.h > 0 ? m.h : 1) * (m.d > 0 ? m.d : 1) * (m.c > 0 ? m.c : 1);
        if (cudaMalloc(&dst, n * 4) != cudaSuccess) return -100;
        return cudaMemcpy(dst, m.data, n * 4, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : S2_ERR_CUDA;
    };
    int r = put(e.data, e.d_data);
    if (r == 0) r = put(e.gamma, e.d_gamma);
    if (r == 0) r = put(e.beta, e.d_beta);
    return r;
}

Extractor Net::create_extractor() const
{
    return Extractor(this);
}

// ---------------------------------------------------------------- Extractor
Extractor::Extractor(const Net* n) : net(n), slots(n->blob_names.size()), mem(n->blob_names.size())
{
    for (size_t i = 0; i < slots.size(); i++) slots[i].pending = n->blob_consumers[i];
}

Extractor::Extractor(Extractor&& o) : net(o.net), slots(std::move(o.slots)), mem(std::move(o.mem)) {}

Extractor::~Extractor() {}

int Extractor::alloc(Slot& s, int w, int h)
{
    std::shared_ptr<void> p = net->blob_alloc((size_t)w * h * 4);
    if (!p) return -100;
    const size_t idx = &s - slots.data();
    mem[idx] = p;
    s.b.data = p.get();
    s.b.w = w;
    s.b.h = h;
    s.b.ld = w;
    s.b.dtype = S2_DTYPE_F32;
    s.owned = true;
    return 0;
}

void Extractor::release(int blob)
{
    Slot& s = slots[blob];
    if (s.input || s.pinned || !s.b.data) return;
    mem[blob].reset();
    s.b = CudaBlob();
    s.owned = false;
}

int Extractor::input(const char* name, const ncnn::Mat& in)
{
    const int b = net->blob_index(name);
    if (b < 0 || in.empty() || in.elemsize != 4 || (in.dims != 1 && in.dims != 2)) return -1;
    Slot& s = slots[b];
    const int h = in.dims == 1 ? 1 : in.h;
    if (alloc(s, in.w, h) != 0) return -100;
    if (cudaMemcpy(s.b.data, in.data, (size_t)in.w * h * 4, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
    s.input = true;
    return 0;
}

int Extractor::input_cuda(const char* name, const CudaBlob& in)
{
    const int b = net->blob_index(name);
    if (b < 0 || !in.data || in.dtype != S2_DTYPE_F32 || in.w <= 0 || in.h <= 0 || in.ld != in.w) return -1;
    Slot& s = slots[b];
    s.b = in;
    s.owned = false;
    s.input = true;
    return 0;
}

int Extractor::extract(const char* name, ncnn::Mat& out)
{
    CudaBlob b;
    int r = extract_cuda(name, b);
    if (r != 0) return r;
    r = s2_status(layer_context());
    if (r != 0) return r;
    out.create(b.w, b.h, (size_t)4u);
    if (out.empty()) return -100;
    return cudaMemcpy(out.data, b.data, (size_t)b.w * b.h * 4, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

int Extractor::extract_cuda(const char* name, CudaBlob& out)
{
    const int b = net->blob_index(name);
    if (b < 0 || !net->model_loaded) return -1;
    const int r = compute(b, 0);
    if (r != 0) return r;
    slots[b].pinned = true;
    out = slots[b].b;
    return 0;
}

int Extractor::compute(int blob, int depth)
{
    if (slots[blob].b.data) return 0;
    if (depth > 100000) return -1;
    const int li = net->blob_producer[blob];
    if (net->layers[li].type == "Input") return -1; // an input that was never bound
    return run_layer(li, depth + 1);
}

int Extractor::run_layer(int li, int depth)
{
    const Net::Entry& e = net->layers[li];
    const AdaptiveWindowAttention* awa = dynamic_cast<const AdaptiveWindowAttention*>(e.layer);
    // the attention's device forward reads only its qkv blobs: the shape and
    // text-length blobs come from the runtime state, as on the reference's
    // GPU path (adaptive_window_attention.cpp:1059-1114)
    const size_t needed = awa ? (e.bottoms.size() == 8 ? 6 : 2) : e.bottoms.size();
    for (size_t k = 0; k < needed && k < e.bottoms.size(); k++)
    {
        const int r = compute(e.bottoms[k], depth);
        if (r != 0) return r;
    }
    s2_context* ctx = layer_context();
    if (!ctx) return S2_ERR_DEVICE;
    int r = 0;
    auto in = [&](int k) -> const CudaBlob& { return slots[e.bottoms[k]].b; };
    auto top = [&](int k) -> Slot& { return slots[e.tops[k]]; };
    if (e.type == "Split")
    {
        for (size_t k = 0; k < e.tops.size(); k++)
        {
            top(k).b = in(0);
            mem[e.tops[k]] = mem[e.bottoms[0]]; // shares the memory (or borrows an input)
            top(k).pending = net->blob_consumers[e.tops[k]];
        }
    }
    else if (e.type == "MemoryData")
    {
        if ((r = net->upload(e)) != 0) return r;
        Slot& t = top(0);
        t.b.data = e.d_data; // owned by the net
        t.b.w = e.w;
        t.b.h = (e.h > 0 ? e.h : 1) * (e.c > 0 ? e.c : 1);
        t.b.ld = e.w;
        t.b.dtype = S2_DTYPE_F32;
        t.input = true; // never released by the extractor
    }
    else if (e.type == "BinaryOp")
    {
        CudaBlob a = in(0), b;
        std::shared_ptr<void> scalar_mem;
        if (e.with_scalar)
        {
            std::vector<float> v((size_t)a.w, e.scalar);
            scalar_mem = net->blob_alloc((size_t)a.w * 4);
            if (!scalar_mem) return -100;
            if (cudaMemcpy(scalar_mem.get(), v.data(), v.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) return -1;
            b.data = scalar_mem.get();
            b.w = a.w;
            b.h = 1;
        }
        else
            b = in(1);
        if (a.h == 1 && b.h > 1 && (e.op == S2_BINARY_ADD || e.op == S2_BINARY_MUL)) std::swap(a, b);
        if (a.w != b.w || (b.h != 1 && b.h != a.h)) return -1;
        if ((r = alloc(top(0), a.w, a.h)) != 0) return r;
        r = s2_binary_op(ctx, e.op, a.h, a.w, static_cast<const float*>(a.data), static_cast<const float*>(b.data),
                         b.h, static_cast<float*>(top(0).b.data));
        if (r == 0 && scalar_mem) r = s2_status(ctx); // the scalar row is freed next
    }
    else if (e.type == "RMSNorm" || e.type == "LayerNorm")
    {
        const CudaBlob& x = in(0);
        if (e.affine && e.affine_size != x.w) return -1;
        if ((r = net->upload(e)) != 0) return r;
        if ((r = alloc(top(0), x.w, x.h)) != 0) return r;
        r = s2_norm_f32(ctx, e.type == "LayerNorm", x.h, x.w, static_cast<const float*>(x.data), e.eps,
                        e.affine ? e.d_gamma : nullptr, e.affine ? e.d_beta : nullptr,
                        static_cast<float*>(top(0).b.data));
    }
    else if (e.type == "GELU")
    {
        const CudaBlob& x = in(0);
        if ((r = alloc(top(0), x.w, x.h)) != 0) return r;
        r = s2_gelu_f32(ctx, e.fast, (int64_t)x.w * x.h, static_cast<const float*>(x.data),
                        static_cast<float*>(top(0).b.data));
    }
    else if (const SharedLinear* sl = dynamic_cast<const SharedLinear*>(e.layer))
    {
        // bf16 operands for the tensor cores, fp32 outputs for the graph
        if (e.bottoms.size() != 2 || e.tops.size() != 2) return -1;
        std::vector<CudaBlob> bot(2), tp(2);
        std::shared_ptr<void> tmp[2];
        for (int k = 0; k < 2; k++)
        {
            const CudaBlob& x = in(k);
            tmp[k] = net->blob_alloc((size_t)x.w * x.h * 2);
            if (!tmp[k]) return -100;
            if ((r = s2_convert_f32_bf16(ctx, static_cast<const float*>(x.data), tmp[k].get(), (int64_t)x.w * x.h)) != 0)
                return r;
            bot[k] = x;
            bot[k].data = tmp[k].get();
            bot[k].dtype = S2_DTYPE_BF16;
        }
        const int n_out = e.pd.get(0, 0); // num_output
        for (int k = 0; k < 2; k++)
        {
            if ((r = alloc(top(k), n_out, in(k).h)) != 0) return r;
            tp[k] = top(k).b;
        }
        r = sl->forward_cuda(bot, tp);
        if (r == 0) r = s2_status(ctx); // the bf16 copies are freed next
    }
    else if (awa)
    {
        const size_t nq = needed;
        if ((e.bottoms.size() != 4 && e.bottoms.size() != 8) || e.tops.size() != 2) return -1;
        std::vector<CudaBlob> bot(nq), tp(2);
        for (size_t k = 0; k < nq; k++) bot[k] = in((int)k);
        const int inner = e.pd.get(0, 0) * e.pd.get(1, 0);
        if ((r = alloc(top(0), inner, in(0).h)) != 0) return r;
        if ((r = alloc(top(1), inner, in(nq == 6 ? 3 : 1).h)) != 0) return r;
        tp[0] = top(0).b;
        tp[1] = top(1).b;
        r = awa->forward_cuda(bot, tp);
    }
    else if (e.layer)
    {
        // another registered custom layer: its host forward
        if ((r = s2_status(ctx)) != 0) return r;
        std::vector<ncnn::Mat> bot(e.bottoms.size()), tp(e.tops.size());
        for (size_t k = 0; k < e.bottoms.size(); k++)
        {
            const CudaBlob& x = in((int)k);
            bot[k].create(x.w, x.h, (size_t)4u);
            if (bot[k].empty() ||
                cudaMemcpy(bot[k].data, x.data, (size_t)x.w * x.h * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                return -1;
        }
        ncnn::Option opt;
        if ((r = e.layer->forward(bot, tp, opt)) != 0) return r;
        for (size_t k = 0; k < e.tops.size(); k++)
        {
            const ncnn::Mat& m = tp[k];
            const int h = m.dims == 1 ? 1 : m.h;
            if (m.empty() || m.elemsize != 4 || m.dims > 2) return -1;
            if ((r = alloc(top((int)k), m.w, h)) != 0) return r;
            if (cudaMemcpy(top((int)k).b.data, m.data, (size_t)m.w * h * 4, cudaMemcpyHostToDevice) != cudaSuccess)
                return -1;
        }
    }
    else
        return -1;
    if (r != 0) return r;
    for (int t : e.tops)
        if (e.type != "Split") slots[t].pending = net->blob_consumers[t];
    // light mode: a bottom is released once its last consumer has run
    for (size_t k = 0; k < needed && k < e.bottoms.size(); k++)
        if (--slots[e.bottoms[k]].pending <= 0) release(e.bottoms[k]);
    return 0;
}

} // namespace seedvr2
