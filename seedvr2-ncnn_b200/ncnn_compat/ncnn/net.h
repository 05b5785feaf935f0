// Subset of Tencent/ncnn's Net: custom-layer registration and creation.
#pragma once

#include <string>
#include <vector>

#include "layer.h"

namespace ncnn
{

class Net
{
public:
    struct Registered
    {
        std::string type;
        layer_creator_func creator;
        layer_destroyer_func destroyer;
        void* userdata;
    };

    int register_custom_layer(const char* type, layer_creator_func creator, layer_destroyer_func destroyer = 0,
                              void* userdata = 0)
    {
        for (size_t i = 0; i < layers.size(); i++)
            if (layers[i].type == type)
            {
                layers[i].creator = creator;
                layers[i].destroyer = destroyer;
                layers[i].userdata = userdata;
                return 0;
            }
        Registered r = {type, creator, destroyer, userdata};
        layers.push_back(r);
        return 0;
    }

    Layer* create_custom_layer(const char* type) const
    {
        for (size_t i = 0; i < layers.size(); i++)
            if (layers[i].type == type)
                return layers[i].creator(layers[i].userdata);
        return 0;
    }

    void destroy_custom_layer(const char* type, Layer* layer) const
    {
        for (size_t i = 0; i < layers.size(); i++)
            if (layers[i].type == type && layers[i].destroyer)
            {
                layers[i].destroyer(layer, layers[i].userdata);
                return;
            }
        delete layer;
    }

    std::vector<Registered> layers;
};

} // namespace ncnn
