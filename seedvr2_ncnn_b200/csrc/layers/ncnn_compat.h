// The subset of the ncnn API that the SeedVR2 custom layers are written
// against (ncnn::Mat, ParamDict, ModelBin, Option, Layer).  Building inside an
// ncnn tree (S2_WITH_NCNN defined) uses ncnn's own headers instead; this file
// only lets the layer classes build and run where ncnn is not installed.
//
// Semantics follow ncnn's public API: Mat is a reference-counted host blob of
// dims/w/h/d/c (n = 1: one sample) whose 3-D and 4-D channel steps are
// rounded up to 16 bytes; ModelBin::load(w, 1) reads w raw fp32 values;
// ParamDict maps integer ids to int/float values.
#pragma once

#ifdef S2_WITH_NCNN
#include <layer.h>
#include <modelbin.h>
#include <paramdict.h>
#else

#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <map>
#include <vector>

namespace ncnn {

class Allocator
{
public:
    virtual ~Allocator() {}
};

class Mat
{
public:
    Mat() {}
    Mat(int w, size_t es = 4u) { create(w, es); }
    Mat(int w, int h, size_t es = 4u) { create(w, h, es); }
    Mat(int w, int h, int c, size_t es = 4u) { create(w, h, c, es); }
    Mat(int w, int h, int d, int c, size_t es = 4u) { create(w, h, d, c, es); }
    Mat(const Mat& m) { assign(m); }
    Mat& operator=(const Mat& m)
    {
        if (this != &m)
        {
            release();
            assign(m);
        }
        return *this;
    }
    ~Mat() { release(); }

    void create(int _w, size_t es = 4u, Allocator* = 0) { shape(1, _w, 1, 1, 1, es); }
    void create(int _w, int _h, size_t es = 4u, Allocator* = 0) { shape(2, _w, _h, 1, 1, es); }
    void create(int _w, int _h, int _c, size_t es = 4u, Allocator* = 0) { shape(3, _w, _h, 1, _c, es); }
    void create(int _w, int _h, int _d, int _c, size_t es = 4u, Allocator* = 0) { shape(4, _w, _h, _d, _c, es); }
    // the batched form of the pinned ncnn (elempack 1, n 1 here)
    void create(int _w, int _h, int _d, int _c, size_t es, int, int, Allocator* = 0) { shape(4, _w, _h, _d, _c, es); }
    bool empty() const { return data == 0 || total() == 0; }
    size_t total() const { return cstep * c; }
    float* row(int y) { return (float*)((unsigned char*)data + (size_t)w * y * elemsize); }
    const float* row(int y) const { return (const float*)((const unsigned char*)data + (size_t)w * y * elemsize); }
    template <typename T> operator T*() { return (T*)data; }
    template <typename T> operator const T*() const { return (const T*)data; }
    void fill(float v)
    {
        for (size_t i = 0; i < total(); i++) ((float*)data)[i] = v;
    }
    Mat reshape(int _w, int _h) const
    {
        Mat m(*this);
        if ((size_t)_w * _h != (size_t)w * h * d * c) return Mat();
        m.dims = 2;
        m.w = _w;
        m.h = _h;
        m.d = 1;
        m.c = 1;
        m.cstep = (size_t)_w * _h;
        return m;
    }

    void* data = 0;
    int* refcount = 0;
    size_t elemsize = 0;
    int elempack = 0;
    Allocator* allocator = 0;
    int dims = 0, w = 0, h = 0, d = 1, c = 0, n = 1;
    size_t cstep = 0;

private:
    void shape(int _dims, int _w, int _h, int _d, int _c, size_t es)
    {
        release();
        dims = _dims;
        w = _w;
        h = _h;
        d = _d;
        c = _c;
        elemsize = es;
        elempack = 1;
        const size_t plane = (size_t)w * h * d * es;
        cstep = (dims >= 3 ? ((plane + 15) & ~(size_t)15) : plane) / es;
        const size_t bytes = total() * es;
        if (!bytes) return;
        data = std::malloc(bytes + 64);
        refcount = new int(1);
    }
    void assign(const Mat& m)
    {
        data = m.data;
        refcount = m.refcount;
        if (refcount) ++*refcount;
        elemsize = m.elemsize;
        elempack = m.elempack;
        allocator = m.allocator;
        dims = m.dims;
        w = m.w;
        h = m.h;
        d = m.d;
        c = m.c;
        n = m.n;
        cstep = m.cstep;
    }
    void release()
    {
        if (refcount && --*refcount == 0)
        {
            std::free(data);
            delete refcount;
        }
        data = 0;
        refcount = 0;
        dims = w = h = c = 0;
        d = n = 1;
        cstep = 0;
    }
};

class ParamDict
{
public:
    int get(int id, int def) const
    {
        auto it = v.find(id);
        return it == v.end() ? def : (it->second.is_f ? (int)it->second.f : it->second.i);
    }
    float get(int id, float def) const
    {
        auto it = v.find(id);
        return it == v.end() ? def : (it->second.is_f ? it->second.f : (float)it->second.i);
    }
    void set(int id, int x) { v[id] = {false, x, 0.f}; }
    void set(int id, float x) { v[id] = {true, 0, x}; }

private:
    struct E
    {
        bool is_f;
        int i;
        float f;
    };
    std::map<int, E> v;
};

class ModelBin
{
public:
    virtual ~ModelBin() {}
    virtual Mat load(int w, int type) const = 0;
};

class ModelBinFromMatArray : public ModelBin
{
public:
    explicit ModelBinFromMatArray(const Mat* w) : weights(w) {}
    virtual Mat load(int, int) const { return weights[cursor++]; }

private:
    const Mat* weights;
    mutable int cursor = 0;
};

class Option
{
public:
    Allocator* blob_allocator = 0;
    Allocator* workspace_allocator = 0;
    int num_threads = 1;
};

class Layer
{
public:
    virtual ~Layer() {}
    virtual int load_param(const ParamDict&) { return 0; }
    virtual int load_model(const ModelBin&) { return 0; }
    virtual int create_pipeline(const Option&) { return 0; }
    virtual int destroy_pipeline(const Option&) { return 0; }
    virtual int forward(const std::vector<Mat>&, std::vector<Mat>&, const Option&) const { return -1; }
    virtual int forward(const Mat&, Mat&, const Option&) const { return -1; }
    bool one_blob_only = false;
    bool support_inplace = false;
    void* userdata = 0;
};

} // namespace ncnn
#endif
