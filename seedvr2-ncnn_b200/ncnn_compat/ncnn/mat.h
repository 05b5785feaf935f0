// Subset of Tencent/ncnn's Mat API used by the SeedVR2 AWA layer classes:
// refcounted storage, cstep aligned to 16 bytes for dims >= 3, channel() /
// row() / depth() / batch() views aliasing the parent. The AWA layers are
// compiled against real ncnn in an ncnn build; this subset lets them build and
// run standalone (the reference's ncnn submodule is empty). The parity oracle
// compiles the reference's own CPU forward against the same headers.
//
// Batched Mats (n > 1, the NCNN_BATCH layouts) keep each batch item's storage
// on a 4 KiB boundary: nstep is cstep * c rounded up to 4096 bytes, so a
// batch stride is not in general c channel strides.
#pragma once

#include <cstddef>
#include <cstdlib>
#include <cstring>

namespace ncnn
{

class Allocator;

class Mat
{
public:
    Mat() {}
    Mat(int _w, size_t _elemsize, Allocator* _allocator = 0) { create(_w, _elemsize, _allocator); }
    Mat(int _w, int _h, size_t _elemsize, Allocator* _allocator = 0) { create(_w, _h, _elemsize, _allocator); }
    Mat(int _w, int _h, int _c, size_t _elemsize, Allocator* _allocator = 0)
    {
        create(_w, _h, _c, _elemsize, _allocator);
    }
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

    void create(int _w, size_t _elemsize, Allocator* = 0) { create_impl(1, _w, 1, 1, 1, _elemsize, 1, 1); }
    void create(int _w, int _h, size_t _elemsize, Allocator* = 0) { create_impl(2, _w, _h, 1, 1, _elemsize, 1, 1); }
    void create(int _w, int _h, int _c, size_t _elemsize, Allocator* = 0)
    {
        create_impl(3, _w, _h, 1, _c, _elemsize, 1, 1);
    }
    void create(int _w, int _h, int _d, int _c, size_t _elemsize, Allocator* = 0)
    {
        create_impl(4, _w, _h, _d, _c, _elemsize, 1, 1);
    }
    // Batched forms used under NCNN_BATCH: (w, h, c, elemsize, elempack, n) and
    // (w, h, d, c, elemsize, elempack, n).
    void create(int _w, int _h, int _c, size_t _elemsize, int _elempack, int _n, Allocator* = 0)
    {
        create_impl(3, _w, _h, 1, _c, _elemsize, _elempack, _n);
    }
    void create(int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, int _n, Allocator* = 0)
    {
        create_impl(4, _w, _h, _d, _c, _elemsize, _elempack, _n);
    }

    bool empty() const { return data == 0 || total() == 0; }
    size_t total() const { return cstep * c * n; }

    void fill(float v)
    {
        float* p = (float*)data;
        for (size_t i = 0; i < total(); i++)
            p[i] = v;
    }

    // dims 3 -> a (w, h) plane; dims 4 -> a (w, h, c=d) volume, as in ncnn.
    Mat channel(int _c)
    {
        Mat m = view();
        m.data = (unsigned char*)data + cstep * _c * elemsize;
        m.n = 1;
        m.d = 1;
        m.cstep = (size_t)w * h;
        if (dims == 4)
        {
            m.dims = 3;
            m.c = d;
        }
        else
        {
            m.dims = 2;
            m.c = 1;
        }
        m.nstep = m.cstep * m.c;
        return m;
    }
    const Mat channel(int _c) const { return const_cast<Mat*>(this)->channel(_c); }

    Mat depth(int z)
    {
        Mat m = view();
        m.dims = 2;
        m.c = 1;
        m.d = 1;
        m.n = 1;
        m.data = (unsigned char*)data + (size_t)w * h * z * elemsize;
        m.cstep = (size_t)w * h;
        return m;
    }
    const Mat depth(int z) const { return const_cast<Mat*>(this)->depth(z); }

    Mat batch(int b)
    {
        Mat m = view();
        m.n = 1;
        m.data = (unsigned char*)data + nstep * b * elemsize;
        return m;
    }
    const Mat batch(int b) const { return const_cast<Mat*>(this)->batch(b); }

    float* row(int y) { return (float*)((unsigned char*)data + (size_t)w * y * elemsize); }
    const float* row(int y) const { return (const float*)((const unsigned char*)data + (size_t)w * y * elemsize); }

    float& operator[](size_t i) { return ((float*)data)[i]; }
    const float& operator[](size_t i) const { return ((const float*)data)[i]; }

    void* data = 0;
    int* refcount = 0;
    size_t elemsize = 0;
    int elempack = 0;
    Allocator* allocator = 0;
    int dims = 0;
    int w = 0;
    int h = 0;
    int d = 0;
    int c = 0;
    int n = 1;
    size_t cstep = 0;
    size_t nstep = 0;

private:
    Mat view() const
    {
        Mat m;
        m.data = data;
        m.refcount = 0;  // views do not own storage
        m.elemsize = elemsize;
        m.elempack = elempack;
        m.dims = dims;
        m.w = w;
        m.h = h;
        m.d = d;
        m.c = c;
        m.n = n;
        m.cstep = cstep;
        m.nstep = nstep;
        return m;
    }

    void assign(const Mat& m)
    {
        data = m.data;
        refcount = m.refcount;
        if (refcount)
            ++*refcount;
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
        nstep = m.nstep;
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
        dims = w = h = d = c = 0;
        n = 1;
        cstep = nstep = 0;
        elemsize = 0;
        elempack = 0;
    }

    static size_t align16(size_t bytes) { return (bytes + 15) & ~(size_t)15; }

    void create_impl(int _dims, int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, int _n)
    {
        release();
        dims = _dims;
        w = _w;
        h = _h;
        d = _d;
        c = _c;
        n = _n;
        elemsize = _elemsize;
        elempack = _elempack;
        if (dims >= 3)
            cstep = align16((size_t)w * h * d * elemsize) / elemsize;
        else
            cstep = (size_t)w * h;
        nstep = cstep * c;
        if (n > 1)
            nstep = ((nstep * elemsize + 4095) & ~(size_t)4095) / elemsize;
        const size_t bytes = align16(nstep * n * elemsize);
        if (bytes == 0)
            return;
        data = std::calloc(1, bytes + 64);
        refcount = new int(1);
    }
};

} // namespace ncnn
