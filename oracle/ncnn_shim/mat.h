// Clean-room restatement of the subset of the ncnn::Mat API that the
// reference's CPU layer code (src/seedvr2/adaptive_window_attention.cpp,
// src/seedvr2/shared_linear.cpp and src/seedvr2/decomposed_conv3d.cpp,
// compiled with NCNN_VULKAN=0) calls.
//
// TEST INFRASTRUCTURE ONLY.  This header exists so that the reference's own
// layer sources compile unmodified into oracle/_ref; it is never part of the
// shipped library.  Semantics follow the public ncnn documentation:
//   * dims/w/h/c/elemsize/elempack describe the blob;
//   * 3-D and 4-D blobs store each channel (w x h, or w x h x d) at a
//     16-byte aligned stride (cstep); n is the batch count (always 1 here);
//   * storage is reference counted and shared by copies and views.
#ifndef S2_ORACLE_NCNN_SHIM_MAT_H
#define S2_ORACLE_NCNN_SHIM_MAT_H

#include <cstddef>
#include <cstdlib>
#include <cstring>

#ifndef NCNN_VULKAN
#define NCNN_VULKAN 0
#endif

namespace ncnn {

class Allocator
{
public:
    virtual ~Allocator() {}
};

class Mat
{
public:
    Mat() { init_empty(); }
    explicit Mat(int _w, size_t _elemsize = 4u, Allocator* a = 0) { init_empty(); create(_w, _elemsize, a); }
    Mat(int _w, int _h, size_t _elemsize = 4u, Allocator* a = 0) { init_empty(); create(_w, _h, _elemsize, a); }
    Mat(int _w, int _h, int _c, size_t _elemsize = 4u, Allocator* a = 0) { init_empty(); create(_w, _h, _c, _elemsize, a); }
    Mat(int _w, int _h, int _c, size_t _elemsize, int _elempack, Allocator* a)
    {
        init_empty();
        create(_w, _h, _c, _elemsize, a);
        elempack = _elempack;
    }
    Mat(int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, int _n, Allocator* a = 0)
    {
        init_empty();
        create(_w, _h, _d, _c, _elemsize, _elempack, _n, a);
    }
    // External-data 1-D view (not owned).
    Mat(int _w, void* _data, size_t _elemsize = 4u, Allocator* a = 0)
    {
        init_empty();
        data = _data;
        elemsize = _elemsize;
        elempack = 1;
        allocator = a;
        dims = 1;
        w = _w;
        h = d = c = 1;
        cstep = (size_t)w;
    }
    Mat(const Mat& m) : data(m.data), refcount(m.refcount), elemsize(m.elemsize), elempack(m.elempack),
                        allocator(m.allocator), dims(m.dims), w(m.w), h(m.h), d(m.d), c(m.c), n(m.n), cstep(m.cstep)
    {
        if (refcount) ++*refcount;
    }
    ~Mat() { release(); }

    Mat& operator=(const Mat& m)
    {
        if (this == &m) return *this;
        if (m.refcount) ++*m.refcount;
        release();
        data = m.data;
        refcount = m.refcount;
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
        return *this;
    }

    void create(int _w, size_t _elemsize = 4u, Allocator* a = 0)
    {
        release();
        elemsize = _elemsize;
        elempack = 1;
        allocator = a;
        dims = 1;
        w = _w;
        h = d = c = 1;
        cstep = (size_t)w;
        allocate();
    }
    void create(int _w, int _h, size_t _elemsize = 4u, Allocator* a = 0)
    {
        release();
        elemsize = _elemsize;
        elempack = 1;
        allocator = a;
        dims = 2;
        w = _w;
        h = _h;
        d = c = 1;
        cstep = (size_t)w * h;
        allocate();
    }
    void create(int _w, int _h, int _c, size_t _elemsize = 4u, Allocator* a = 0)
    {
        release();
        elemsize = _elemsize;
        elempack = 1;
        allocator = a;
        dims = 3;
        w = _w;
        h = _h;
        d = 1;
        c = _c;
        const size_t bytes = (size_t)w * h * elemsize;
        cstep = ((bytes + 15) & ~(size_t)15) / elemsize;
        allocate();
    }

    // 4-D: w x h x d per channel (d frames), 16-byte aligned channel stride
    void create(int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, int _n, Allocator* a = 0)
    {
        release();
        elemsize = _elemsize;
        elempack = _elempack;
        allocator = a;
        dims = 4;
        w = _w;
        h = _h;
        d = _d;
        c = _c;
        n = _n;
        const size_t bytes = (size_t)w * h * d * elemsize;
        cstep = ((bytes + 15) & ~(size_t)15) / elemsize;
        allocate();
    }

    // ncnn's 4-D create(w, h, d, c[, elemsize, allocator]): pack 1, n 1
    void create(int _w, int _h, int _d, int _c, size_t _elemsize = 4u, Allocator* a = 0)
    {
        create(_w, _h, _d, _c, _elemsize, 1, 1, a);
    }

    void fill(float v)
    {
        float* p = (float*)data;
        const size_t n = total();
        for (size_t i = 0; i < n; i++) p[i] = v;
    }

    Mat clone(Allocator* a = 0) const
    {
        Mat m;
        if (empty()) return m;
        if (dims == 1) m.create(w, elemsize, a);
        else if (dims == 2) m.create(w, h, elemsize, a);
        else m.create(w, h, c, elemsize, a);
        std::memcpy(m.data, data, total() * elemsize);
        return m;
    }

    // Re-shapes a contiguous blob; shares storage.
    Mat reshape(int _w, Allocator* a = 0) const
    {
        (void)a;
        if ((size_t)_w != (size_t)w * h * c) return Mat();
        Mat m = *this;
        m.dims = 1;
        m.w = _w;
        m.h = m.c = m.d = 1;
        m.cstep = (size_t)_w;
        return m;
    }
    Mat reshape(int _w, int _h, Allocator* a = 0) const
    {
        (void)a;
        if ((size_t)_w * _h != (size_t)w * h * c) return Mat();
        if (dims == 3 && cstep != (size_t)w * h) return Mat();
        Mat m = *this;
        m.dims = 2;
        m.w = _w;
        m.h = _h;
        m.c = m.d = 1;
        m.cstep = (size_t)_w * _h;
        return m;
    }

    bool empty() const { return data == 0 || total() == 0; }
    size_t total() const { return cstep * c; }

    // channel _c: a w x h view (3-D blob) or a w x h x d view (4-D blob)
    Mat channel(int _c)
    {
        Mat m(w, h, (unsigned char*)data + cstep * _c * elemsize, elemsize);
        if (dims == 4) m.set_depth(d);
        return m;
    }
    const Mat channel(int _c) const
    {
        Mat m(w, h, (unsigned char*)data + cstep * _c * elemsize, elemsize);
        if (dims == 4) m.set_depth(d);
        return m;
    }
    // frame z of a w x h x d channel view: a w x h view
    Mat depth(int z)
    {
        Mat m(w, h, (unsigned char*)data + (size_t)w * h * z * elemsize, elemsize);
        return m;
    }
    const Mat depth(int z) const
    {
        Mat m(w, h, (unsigned char*)data + (size_t)w * h * z * elemsize, elemsize);
        return m;
    }

    float* row(int y) { return (float*)((unsigned char*)data + (size_t)w * y * elemsize); }
    const float* row(int y) const { return (const float*)((unsigned char*)data + (size_t)w * y * elemsize); }
    template <typename T> T* row(int y) { return (T*)((unsigned char*)data + (size_t)w * y * elemsize); }
    template <typename T> const T* row(int y) const { return (const T*)((unsigned char*)data + (size_t)w * y * elemsize); }

    Mat row_range(int y, int rows)
    {
        Mat m(w, rows, (unsigned char*)data + (size_t)w * y * elemsize, elemsize);
        return m;
    }

    template <typename T> operator T*() { return (T*)data; }
    template <typename T> operator const T*() const { return (const T*)data; }
    float& operator[](size_t i) { return ((float*)data)[i]; }
    const float& operator[](size_t i) const { return ((const float*)data)[i]; }

    void release()
    {
        if (refcount && --*refcount == 0)
        {
            std::free(data);
            delete refcount;
        }
        data = 0;
        refcount = 0;
        dims = 0;
        w = h = d = c = 0;
        n = 1;
        cstep = 0;
        elemsize = 0;
        elempack = 0;
    }

    void* data;
    int* refcount;
    size_t elemsize;
    int elempack;
    Allocator* allocator;
    int dims;
    int w;
    int h;
    int d;
    int c;
    int n;
    size_t cstep;

private:
    void set_depth(int _d)
    {
        dims = 3;
        d = _d;
        cstep = (size_t)w * h * d;
    }
    // 2-D external view used by channel()/row_range().
    Mat(int _w, int _h, void* _data, size_t _elemsize)
    {
        init_empty();
        data = _data;
        elemsize = _elemsize;
        elempack = 1;
        dims = 2;
        w = _w;
        h = _h;
        d = c = 1;
        cstep = (size_t)w * h;
    }
    void init_empty()
    {
        data = 0;
        refcount = 0;
        elemsize = 0;
        elempack = 0;
        allocator = 0;
        dims = 0;
        w = h = d = c = 0;
        n = 1;
        cstep = 0;
    }
    void allocate()
    {
        const size_t bytes = total() * elemsize;
        if (bytes == 0) return;
        // 64-byte aligned, padded like ncnn (which over-allocates a little).
        data = std::aligned_alloc(64, ((bytes + 63) & ~(size_t)63) + 64);
        if (!data) return;
        refcount = new int(1);
    }
};

} // namespace ncnn

#endif
