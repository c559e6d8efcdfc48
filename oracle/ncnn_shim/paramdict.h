// Clean-room ParamDict subset (id -> int/float) for compiling the reference's
// layer sources into the CPU oracle.  TEST INFRASTRUCTURE ONLY.
#ifndef S2_ORACLE_NCNN_SHIM_PARAMDICT_H
#define S2_ORACLE_NCNN_SHIM_PARAMDICT_H

#include <map>

#include "mat.h"

namespace ncnn {

class ParamDict
{
public:
    int get(int id, int def) const
    {
        std::map<int, Entry>::const_iterator it = values.find(id);
        if (it == values.end()) return def;
        return it->second.is_float ? (int)it->second.f : it->second.i;
    }
    float get(int id, float def) const
    {
        std::map<int, Entry>::const_iterator it = values.find(id);
        if (it == values.end()) return def;
        return it->second.is_float ? it->second.f : (float)it->second.i;
    }
    void set(int id, int v)
    {
        Entry e;
        e.is_float = false;
        e.i = v;
        e.f = 0.f;
        values[id] = e;
    }
    void set(int id, float v)
    {
        Entry e;
        e.is_float = true;
        e.i = 0;
        e.f = v;
        values[id] = e;
    }

private:
    struct Entry
    {
        bool is_float;
        int i;
        float f;
    };
    std::map<int, Entry> values;
};

} // namespace ncnn

#endif
