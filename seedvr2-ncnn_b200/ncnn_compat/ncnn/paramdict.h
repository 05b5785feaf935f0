// Subset of Tencent/ncnn's ParamDict: integer params by id.
#pragma once

#include <map>

namespace ncnn
{

class ParamDict
{
public:
    int get(int id, int def) const
    {
        std::map<int, int>::const_iterator it = ints.find(id);
        return it == ints.end() ? def : it->second;
    }
    void set(int id, int v) { ints[id] = v; }

private:
    std::map<int, int> ints;
};

} // namespace ncnn
