// TEST INFRASTRUCTURE ONLY -- never linked into the product library.
//
// Minimal stand-in for the subset of the ncnn public API (ncnn pinned at
// 81e8cbff upstream; the reference's `ncnn/` submodule is empty and there is no
// network) that the reference's CPU layer sources need in order to compile
// unmodified:
//   src/layers/seedvr2_dit_block.cpp            (NCNN_VULKAN=0)
//   src/layers/dynamic_framewise_spatial_attention.cpp (NCNN_VULKAN=0)
// Only names, signatures and documented semantics of ncnn's public headers are
// mirrored (Mat / Allocator / Option / ParamDict / ModelBin); the code is ours.
// Mat keeps ncnn's memory model: refcounted, row-major, 4-D mats padded per
// channel to a 16-byte aligned `cstep`.
#pragma once

#include <atomic>
#include <cstddef>
#include <cstdlib>
#include <cstring>
#include <vector>

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
    Mat() : data(0), refcount(0), elemsize(0), elempack(0), allocator(0), dims(0), w(0), h(0), d(0), c(0), cstep(0) {}
    Mat(int _w, size_t _elemsize = 4u, Allocator* _a = 0) : Mat() { create(_w, _elemsize, _a); }
    Mat(int _w, int _h, size_t _elemsize = 4u, Allocator* _a = 0) : Mat() { create(_w, _h, _elemsize, _a); }
    Mat(int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, Allocator* _a = 0) : Mat()
    {
        create(_w, _h, _d, _c, _elemsize, _elempack, _a);
    }
    Mat(const Mat& m)
        : data(m.data), refcount(m.refcount), elemsize(m.elemsize), elempack(m.elempack), allocator(m.allocator),
          dims(m.dims), w(m.w), h(m.h), d(m.d), c(m.c), cstep(m.cstep)
    {
        if (refcount) refcount->fetch_add(1);
    }
    ~Mat() { release(); }

    Mat& operator=(const Mat& m)
    {
        if (this == &m) return *this;
        if (m.refcount) m.refcount->fetch_add(1);
        release();
        data = m.data; refcount = m.refcount; elemsize = m.elemsize; elempack = m.elempack;
        allocator = m.allocator; dims = m.dims; w = m.w; h = m.h; d = m.d; c = m.c; cstep = m.cstep;
        return *this;
    }

    void create(int _w, size_t _elemsize = 4u, Allocator* _a = 0) { create_impl(1, _w, 1, 1, 1, _elemsize, 1, _a); }
    void create(int _w, int _h, size_t _elemsize = 4u, Allocator* _a = 0) { create_impl(2, _w, _h, 1, 1, _elemsize, 1, _a); }
    void create(int _w, int _h, size_t _elemsize, int _elempack, Allocator* _a)
    {
        create_impl(2, _w, _h, 1, 1, _elemsize, _elempack, _a);
    }
    void create(int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, Allocator* _a = 0)
    {
        create_impl(4, _w, _h, _d, _c, _elemsize, _elempack, _a);
    }

    void release()
    {
        if (refcount && refcount->fetch_sub(1) == 1)
        {
            std::free(data);
            delete refcount;
        }
        data = 0; refcount = 0; elemsize = 0; elempack = 0; dims = 0; w = h = d = c = 0; cstep = 0;
    }

    bool empty() const { return data == 0 || total() == 0; }
    size_t total() const { return cstep * c; }

    void fill(float v)
    {
        float* p = (float*)data;
        const size_t n = total();
        for (size_t i = 0; i < n; i++) p[i] = v;
    }

    Mat clone(Allocator* _a = 0) const
    {
        if (empty()) return Mat();
        Mat m;
        m.create_impl(dims, w, h, d, c, elemsize, elempack, _a);
        std::memcpy(m.data, data, total() * elemsize);
        return m;
    }

    // Non-owning views, as ncnn::Mat::channel / depth / row.
    Mat channel(int _c) const
    {
        Mat m;
        m.data = (unsigned char*)data + cstep * _c * elemsize;
        m.elemsize = elemsize; m.elempack = elempack; m.allocator = allocator;
        m.dims = dims - 1; m.w = w; m.h = h; m.d = d; m.c = 1;
        m.cstep = (size_t)w * h * d;
        if (dims == 4) { m.dims = 3; m.c = d; m.d = 1; m.cstep = (size_t)w * h; }
        return m;
    }
    Mat depth(int z) const
    {
        Mat m;
        m.data = (unsigned char*)data + (size_t)w * h * z * elemsize;
        m.elemsize = elemsize; m.elempack = elempack; m.allocator = allocator;
        m.dims = 2; m.w = w; m.h = h; m.d = 1; m.c = 1; m.cstep = (size_t)w * h;
        return m;
    }

    float* row(int y) { return (float*)((unsigned char*)data + (size_t)w * y * elemsize); }
    const float* row(int y) const { return (const float*)((unsigned char*)data + (size_t)w * y * elemsize); }

    template <typename T>
    operator T*() { return (T*)data; }
    template <typename T>
    operator const T*() const { return (const T*)data; }

    void* data;
    std::atomic<int>* refcount;
    size_t elemsize;
    int elempack;
    Allocator* allocator;
    int dims;
    int w;
    int h;
    int d;
    int c;
    size_t cstep;

private:
    void create_impl(int _dims, int _w, int _h, int _d, int _c, size_t _elemsize, int _elempack, Allocator* _a)
    {
        release();
        dims = _dims; w = _w; h = _h; d = _d; c = _c; elemsize = _elemsize; elempack = _elempack; allocator = _a;
        if (dims <= 2)
            cstep = (size_t)w * h;
        else
            cstep = (((size_t)w * h * d * elemsize + 15) & ~(size_t)15) / elemsize;
        const size_t bytes = total() * elemsize;
        if (bytes == 0) return;
        data = std::calloc(1, (bytes + 63) & ~(size_t)63);
        refcount = new std::atomic<int>(1);
    }
};

class Option
{
public:
    Option() : lightmode(true), num_threads(1), blob_allocator(0), workspace_allocator(0),
               use_vulkan_compute(false), use_packing_layout(false), use_fp16_packed(false),
               use_fp16_storage(false), use_fp16_arithmetic(false) {}
    bool lightmode;
    int num_threads;
    Allocator* blob_allocator;
    Allocator* workspace_allocator;
    bool use_vulkan_compute;
    bool use_packing_layout;
    bool use_fp16_packed;
    bool use_fp16_storage;
    bool use_fp16_arithmetic;
};

class ParamDict
{
public:
    int get(int id, int def) const { return slot(id).kind == 1 ? slot(id).i : def; }
    float get(int id, float def) const { return slot(id).kind == 2 ? slot(id).f : def; }
    Mat get(int id, const Mat& def) const { return slot(id).kind == 3 ? slot(id).m : def; }
    void set(int id, int v) { grow(id); params[id].kind = 1; params[id].i = v; }
    void set(int id, float v) { grow(id); params[id].kind = 2; params[id].f = v; }
    void set(int id, const Mat& v) { grow(id); params[id].kind = 3; params[id].m = v; }

private:
    struct Entry
    {
        int kind = 0;
        int i = 0;
        float f = 0.f;
        Mat m;
    };
    const Entry& slot(int id) const
    {
        static const Entry none;
        return id >= 0 && id < (int)params.size() ? params[id] : none;
    }
    void grow(int id)
    {
        if (id >= (int)params.size()) params.resize(id + 1);
    }
    std::vector<Entry> params;
};

class ModelBin
{
public:
    virtual ~ModelBin() {}
    // type 0 = stored with an element-type tag, 1 = raw fp32 (ncnn semantics);
    // this shim stores everything as fp32.
    virtual Mat load(int w, int type) const = 0;
};

// Serves consecutive fp32 arrays from one flat buffer, in load order.
class ModelBinFromFloats : public ModelBin
{
public:
    ModelBinFromFloats(const float* _data, size_t _count) : data(_data), count(_count), cursor(0) {}
    Mat load(int w, int /*type*/) const override
    {
        if (w <= 0 || cursor + (size_t)w > count) return Mat();
        Mat m(w);
        std::memcpy(m.data, data + cursor, (size_t)w * sizeof(float));
        cursor += (size_t)w;
        return m;
    }
    size_t consumed() const { return cursor; }

private:
    const float* data;
    size_t count;
    mutable size_t cursor;
};

} // namespace ncnn
