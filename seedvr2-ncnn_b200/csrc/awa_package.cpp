// awa_package.cpp -- the model-package side of the AWA library (host only):
// reading the AWA layer lines of an ncnn block graph, the dynamic-template
// rewrite of those lines, SHA-256 and the package manifest check.
//
// Reference behaviour followed:
//   graph reading   ncnn .param text as the exporter writes it
//                   (tools/export_dit_block.py:578-644) and as the layers'
//                   load_param reads its ParamDict (src/awa/awa_layers.cpp:90-114,
//                   867-874)
//   make_dynamic    normalize_dynamic_awa_template (tools/export_dit_block.py:38-124)
//   manifest        validate_manifest, is_hex_hash, safe_manifest_path,
//                   sha256_file (src/model/model_registry.cpp:153-200, 248-362)
#include <algorithm>
#include <cctype>
#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <iterator>
#include <map>
#include <set>
#include <string>
#include <system_error>
#include <vector>

#include "awa_b200.h"
#include "awa_internal.h"
#include "awa_package.h"

namespace
{

using awa::report_error;

// ---------------------------------------------------------------- SHA-256
// FIPS 180-4. The round constants are the first 32 bits of the fractional
// parts of the cube roots of the first 64 primes, the initial hash value the
// same for the square roots of the first 8 primes (sections 4.2.2, 5.3.3);
// both are derived here from that definition with exact integer roots.
using u128 = unsigned __int128;

uint64_t integer_root(u128 n, int k)  // floor(n^(1/k)) for k = 2 or 3
{
    const long double approx = k == 2 ? std::sqrt((long double)n) : std::cbrt((long double)n);
    uint64_t x = (uint64_t)approx;
    auto power = [k](u128 v) { return k == 2 ? v * v : v * v * v; };
    while (x > 0 && power(x) > n)
        x--;
    while (power((u128)x + 1) <= n)
        x++;
    return x;
}

struct ShaTables
{
    uint32_t k[64];
    uint32_t h0[8];
    ShaTables()
    {
        int primes[64];
        int found = 0;
        for (int candidate = 2; found < 64; candidate++)
        {
            bool prime = true;
            for (int j = 0; j < found && primes[j] * primes[j] <= candidate; j++)
                if (candidate % primes[j] == 0)
                {
                    prime = false;
                    break;
                }
            if (prime)
                primes[found++] = candidate;
        }
        for (int i = 0; i < 64; i++)
            k[i] = (uint32_t)integer_root((u128)primes[i] << 96, 3);  // low 32 bits = fraction * 2^32
        for (int i = 0; i < 8; i++)
            h0[i] = (uint32_t)integer_root((u128)primes[i] << 64, 2);
    }
};

const ShaTables& sha_tables()
{
    static const ShaTables tables;
    return tables;
}

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

class Sha256
{
public:
    Sha256()
    {
        std::memcpy(state_, sha_tables().h0, sizeof(state_));
    }

    void update(const unsigned char* data, size_t size)
    {
        total_ += size;
        while (size > 0)
        {
            const size_t take = std::min(size, sizeof(block_) - fill_);
            std::memcpy(block_ + fill_, data, take);
            fill_ += take;
            data += take;
            size -= take;
            if (fill_ == sizeof(block_))
            {
                compress(block_);
                fill_ = 0;
            }
        }
    }

    std::string hex()
    {
        const uint64_t bits = total_ * 8;
        const unsigned char one = 0x80, zero = 0;
        update(&one, 1);
        while (fill_ != 56)
            update(&zero, 1);
        unsigned char length[8];
        for (int i = 0; i < 8; i++)
            length[i] = (unsigned char)(bits >> (56 - 8 * i));
        update(length, 8);
        static const char digits[] = "0123456789abcdef";
        std::string out(64, '0');
        for (int i = 0; i < 8; i++)
            for (int j = 0; j < 8; j++)
                out[i * 8 + j] = digits[(state_[i] >> (28 - 4 * j)) & 0xF];
        return out;
    }

private:
    void compress(const unsigned char* p)
    {
        const uint32_t* k = sha_tables().k;
        uint32_t w[64];
        for (int t = 0; t < 16; t++)
            w[t] = (uint32_t)p[4 * t] << 24 | (uint32_t)p[4 * t + 1] << 16 | (uint32_t)p[4 * t + 2] << 8 | p[4 * t + 3];
        for (int t = 16; t < 64; t++)
        {
            const uint32_t s0 = rotr(w[t - 15], 7) ^ rotr(w[t - 15], 18) ^ (w[t - 15] >> 3);
            const uint32_t s1 = rotr(w[t - 2], 17) ^ rotr(w[t - 2], 19) ^ (w[t - 2] >> 10);
            w[t] = w[t - 16] + s0 + w[t - 7] + s1;
        }
        uint32_t a = state_[0], b = state_[1], c = state_[2], d = state_[3];
        uint32_t e = state_[4], f = state_[5], g = state_[6], h = state_[7];
        for (int t = 0; t < 64; t++)
        {
            const uint32_t t1 = h + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) + k[t] + w[t];
            const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
            h = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        state_[0] += a;
        state_[1] += b;
        state_[2] += c;
        state_[3] += d;
        state_[4] += e;
        state_[5] += f;
        state_[6] += g;
        state_[7] += h;
    }

    uint32_t state_[8];
    unsigned char block_[64];
    size_t fill_ = 0;
    uint64_t total_ = 0;
};

bool sha256_file(const std::filesystem::path& path, std::string& digest, std::string& error)
{
    std::ifstream input(path, std::ios::binary);
    if (!input)
    {
        error = "failed to open model package artifact: " + path.string();
        return false;
    }
    Sha256 hash;
    std::vector<char> buffer(1 << 20);
    while (input)
    {
        input.read(buffer.data(), (std::streamsize)buffer.size());
        const std::streamsize count = input.gcount();
        if (count > 0)
            hash.update(reinterpret_cast<const unsigned char*>(buffer.data()), (size_t)count);
    }
    if (!input.eof())
    {
        error = "failed to read model package artifact: " + path.string();
        return false;
    }
    digest = hash.hex();
    return true;
}

// ---------------------------------------------------------------- .param text
// The exporter's tooling reads graphs with Python's str.splitlines() and
// str.split(); these two follow them for ASCII text.
bool is_space(unsigned char c) { return c == ' ' || (c >= 9 && c <= 13) || (c >= 0x1c && c <= 0x1f); }

std::vector<std::string> split_lines(const char* text, size_t length)
{
    std::vector<std::string> lines;
    size_t begin = 0, i = 0;
    while (i < length)
    {
        const unsigned char c = (unsigned char)text[i];
        const bool boundary = c == '\n' || c == '\r' || c == 0x0b || c == 0x0c || c == 0x1c || c == 0x1d || c == 0x1e;
        if (!boundary)
        {
            i++;
            continue;
        }
        lines.emplace_back(text + begin, i - begin);
        i += (c == '\r' && i + 1 < length && text[i + 1] == '\n') ? 2 : 1;
        begin = i;
    }
    if (begin < length)
        lines.emplace_back(text + begin, length - begin);
    return lines;
}

std::vector<std::string> split_fields(const std::string& line)
{
    std::vector<std::string> fields;
    size_t i = 0;
    while (i < line.size())
    {
        while (i < line.size() && is_space((unsigned char)line[i]))
            i++;
        const size_t begin = i;
        while (i < line.size() && !is_space((unsigned char)line[i]))
            i++;
        if (i > begin)
            fields.emplace_back(line, begin, i - begin);
    }
    return fields;
}

std::string join_fields(const std::vector<std::string>& fields)
{
    std::string out;
    for (size_t i = 0; i < fields.size(); i++)
    {
        if (i)
            out += ' ';
        out += fields[i];
    }
    return out;
}

// Python int() of a token: optional sign, decimal digits, single underscores
// between digits. Values beyond long long saturate (only their sign matters to
// the callers).
bool parse_int(const std::string& s, long long& value)
{
    size_t i = 0;
    bool negative = false;
    if (i < s.size() && (s[i] == '+' || s[i] == '-'))
        negative = s[i++] == '-';
    if (i >= s.size())
        return false;
    long long v = 0;
    bool saturated = false, last_digit = false;
    for (; i < s.size(); i++)
    {
        const char c = s[i];
        if (c == '_')
        {
            if (!last_digit || i + 1 >= s.size())
                return false;
            last_digit = false;
            continue;
        }
        if (c < '0' || c > '9')
            return false;
        last_digit = true;
        if (!saturated)
        {
            if (v > (LLONG_MAX - (c - '0')) / 10)
                saturated = true;
            else
                v = v * 10 + (c - '0');
        }
    }
    if (!last_digit)
        return false;
    if (saturated)
        v = LLONG_MAX;
    value = negative ? -v : v;
    return true;
}

struct Layer
{
    std::vector<std::string> fields;
    int bottoms = 0;
    int tops = 0;
    size_t param_start = 0;
    int line_number = 0;  // 1-based

    const std::string& type() const { return fields[0]; }
    const std::string& name() const { return fields[1]; }
    const std::string& bottom(int i) const { return fields[4 + i]; }
    const std::string& top(int i) const { return fields[4 + bottoms + i]; }
};

// parse_layer of normalize_dynamic_awa_template.
bool parse_layer(const std::string& line, Layer& layer, std::string& error)
{
    layer.fields = split_fields(line);
    if (layer.fields.size() < 4)
    {
        error = "invalid ncnn layer line: " + line;
        return false;
    }
    long long b = 0, t = 0;
    if (!parse_int(layer.fields[2], b) || !parse_int(layer.fields[3], t))
    {
        error = "invalid ncnn blob counts: " + line;
        return false;
    }
    if (b < 0 || t < 0 || b > INT_MAX / 2 || t > INT_MAX / 2 || layer.fields.size() < (size_t)(4 + b + t))
    {
        error = "invalid ncnn blob declaration: " + line;
        return false;
    }
    layer.bottoms = (int)b;
    layer.tops = (int)t;
    layer.param_start = (size_t)(4 + b + t);
    return true;
}

bool is_awa_type(const std::string& type)
{
    return type == "SeedVR2AWAPack" || type == "SeedVR2AWAUnpack" || type == "SeedVR2MMRoPE" ||
           type == "SeedVR2WindowAttention";
}

bool header_ok(const std::vector<std::string>& lines)
{
    return lines.size() >= 2 && lines[0].compare(0, 7, "7767517") == 0;
}

int fail(const std::string& message) { return report_error(AWA_ERR_INVALID, message.c_str()); }

// normalize_dynamic_awa_template on a text; false with error set when the
// reference function raises.
bool make_dynamic(const char* text, size_t length, std::string& out, std::string& error)
{
    const std::vector<std::string> lines = split_lines(text, length);
    if (!header_ok(lines))
    {
        error = "unexpected ncnn param header";
        return false;
    }
    std::vector<std::string> rewritten(lines);
    std::vector<std::string> unpack_video_blobs;
    int awa_layers = 0;
    for (size_t index = 2; index < lines.size(); index++)
    {
        Layer layer;
        if (!parse_layer(lines[index], layer, error))
            return false;
        if (!is_awa_type(layer.type()))
            continue;
        awa_layers++;
        if (layer.type() == "SeedVR2AWAUnpack")
        {
            if (layer.tops != 2)
            {
                error = "SeedVR2AWAUnpack must expose video and text outputs";
                return false;
            }
            unpack_video_blobs.push_back(layer.top(0));
        }
        int position[3] = {-1, -1, -1};
        for (size_t f = layer.param_start; f < layer.fields.size(); f++)
        {
            const std::string& field = layer.fields[f];
            const size_t eq = field.find('=');
            if (eq == std::string::npos)
                continue;
            const std::string key = field.substr(0, eq);
            if (key != "0" && key != "1" && key != "2")
                continue;
            const int k = key[0] - '0';
            if (position[k] >= 0)
            {
                error = "duplicate AWA parameter " + key + " in " + layer.name();
                return false;
            }
            position[k] = (int)f;
        }
        if (position[0] < 0 || position[1] < 0 || position[2] < 0)
        {
            error = "incomplete AWA grid metadata in " + layer.name();
            return false;
        }
        for (int k = 0; k < 3; k++)
            layer.fields[position[k]] = std::to_string(k) + "=-1";
        rewritten[index] = join_fields(layer.fields);
    }
    if (awa_layers == 0)
    {
        error = "no SeedVR2 AWA layers found";
        return false;
    }
    if (unpack_video_blobs.size() != 1)
    {
        error = "expected one SeedVR2AWAUnpack layer, found " + std::to_string(unpack_video_blobs.size());
        return false;
    }
    int reshapes = 0;
    for (size_t index = 2; index < rewritten.size(); index++)
    {
        Layer layer;
        if (!parse_layer(rewritten[index], layer, error))
            return false;
        if (layer.type() != "Reshape" || layer.name() != "reshape_awa_video_batch" || layer.bottoms != 1 ||
            layer.tops != 1 || layer.bottom(0) != unpack_video_blobs[0])
            continue;
        reshapes++;
        int height = -1, found = 0;
        for (size_t f = layer.param_start; f < layer.fields.size(); f++)
            if (layer.fields[f].compare(0, 2, "1=") == 0)
            {
                height = (int)f;
                found++;
            }
        if (found != 1)
        {
            error = "reshape_awa_video_batch must have exactly one height parameter";
            return false;
        }
        layer.fields[height] = "1=-1";
        rewritten[index] = join_fields(layer.fields);
    }
    if (reshapes != 1)
    {
        error = "expected one AWA video batch reshape, found " + std::to_string(reshapes);
        return false;
    }
    out.clear();
    for (const std::string& line : rewritten)
    {
        out += line;
        out += '\n';
    }
    return true;
}

// One AWA line's ParamDict, as load_common and MMRoPE::load_param read it.
struct AwaParams
{
    long long value[9];
    bool present[9];
};

bool read_awa_params(const Layer& layer, AwaParams& p, std::string& error)
{
    for (int i = 0; i < 9; i++)
    {
        p.value[i] = 0;
        p.present[i] = false;
    }
    std::map<long long, bool> seen;
    for (size_t f = layer.param_start; f < layer.fields.size(); f++)
    {
        const std::string& field = layer.fields[f];
        const size_t eq = field.find('=');
        long long id = 0;
        if (eq == std::string::npos || !parse_int(field.substr(0, eq), id) || field.find('_') < eq)
        {
            error = "invalid parameter '" + field + "' in " + layer.name();
            return false;
        }
        if (seen.count(id))
        {
            error = "duplicate AWA parameter " + std::to_string(id) + " in " + layer.name();
            return false;
        }
        seen[id] = true;
        if (id < 0 || id > 8)
            continue;
        long long v = 0;
        const std::string text = field.substr(eq + 1);
        if (!parse_int(text, v) || text.find('_') != std::string::npos || v < INT_MIN || v > INT_MAX)
        {
            error = "parameter " + std::to_string(id) + " of " + layer.name() + " is not an integer: " + text;
            return false;
        }
        p.value[id] = v;
        p.present[id] = true;
    }
    return true;
}

bool check_grid(const Layer& layer, const AwaParams& p, bool& dynamic, std::string& error)
{
    const long long* v = p.value;
    dynamic = v[0] == -1 && v[1] == -1 && v[2] == -1;
    // T*H*W must fit an int; each factor is checked against INT_MAX divided by
    // the others before any product is formed, so nothing can overflow.
    const bool grid_ok = dynamic || (v[0] > 0 && v[1] > 0 && v[2] > 0 && v[0] <= INT_MAX / v[1] &&
                                     v[0] * v[1] <= INT_MAX / v[2]);
    if (!grid_ok || v[3] <= 0 || v[4] <= 0 || v[5] <= 0 || v[6] <= 0)
    {
        error = "invalid AWA grid metadata in " + layer.name() +
                " (ids 0-2 must be all -1 or positive, ids 3-6 positive)";
        return false;
    }
    if (layer.type() == "SeedVR2MMRoPE")
    {
        const long long rope = p.present[8] ? v[8] : 126;
        if (rope <= 0 || rope % 6 != 0)
        {
            error = "invalid rope dimension " + std::to_string(rope) + " in " + layer.name();
            return false;
        }
    }
    return true;
}

struct ChainLayers
{
    int pack = -1, rope = -1, attention = -1, unpack = -1, reshape = -1;
};

int find_chains(const char* text, size_t length, awa_graph_chain* chains, int capacity)
{
    const std::vector<std::string> lines = split_lines(text, length);
    if (lines.empty() || split_fields(lines[0]).empty() || split_fields(lines[0])[0] != "7767517")
        return fail("unexpected ncnn param header");
    if (lines.size() < 2)
        return fail("ncnn param text has no layer/blob count line");
    const std::vector<std::string> counts = split_fields(lines[1]);
    long long layer_count = 0, blob_count = 0;
    if (counts.size() != 2 || !parse_int(counts[0], layer_count) || !parse_int(counts[1], blob_count) ||
        layer_count < 0 || blob_count < 0)
        return fail("invalid ncnn layer/blob count line: " + lines[1]);
    if ((long long)lines.size() - 2 != layer_count)
        return fail("ncnn param declares " + std::to_string(layer_count) + " layers but holds " +
                    std::to_string(lines.size() - 2) + " layer lines");

    std::string error;
    std::vector<Layer> layers(lines.size() - 2);
    std::vector<AwaParams> params(layers.size());
    std::vector<int> packs, unpacks, others;
    for (size_t i = 0; i < layers.size(); i++)
    {
        Layer& layer = layers[i];
        if (!parse_layer(lines[i + 2], layer, error))
            return fail(error);
        layer.line_number = (int)i + 3;
        if (!is_awa_type(layer.type()))
            continue;
        const std::string& type = layer.type();
        const int want_bottoms = type == "SeedVR2AWAPack" ? 2 : 1;
        const int want_tops = (type == "SeedVR2AWAPack" || type == "SeedVR2AWAUnpack") ? 2 : 1;
        if (layer.bottoms != want_bottoms || layer.tops != want_tops)
            return fail(type + " " + layer.name() + " must have " + std::to_string(want_bottoms) + " inputs and " +
                        std::to_string(want_tops) + " outputs");
        bool dynamic = false;
        if (!read_awa_params(layer, params[i], error) || !check_grid(layer, params[i], dynamic, error))
            return fail(error);
        if (type == "SeedVR2AWAPack")
            packs.push_back((int)i);
        else if (type == "SeedVR2AWAUnpack")
            unpacks.push_back((int)i);
        else
            others.push_back((int)i);
    }
    if (packs.empty() && unpacks.empty() && others.empty())
        return 0;
    if (packs.size() != unpacks.size())
        return fail(std::to_string(packs.size()) + " SeedVR2AWAPack layers but " + std::to_string(unpacks.size()) +
                    " SeedVR2AWAUnpack layers");

    std::vector<ChainLayers> chain(packs.size());
    for (size_t k = 0; k < packs.size(); k++)
    {
        if (unpacks[k] < packs[k] || (k + 1 < packs.size() && unpacks[k] > packs[k + 1]))
            return fail("SeedVR2AWAUnpack " + layers[unpacks[k]].name() + " does not close the chain of " +
                        layers[packs[k]].name());
        chain[k].pack = packs[k];
        chain[k].unpack = unpacks[k];
    }
    for (int i : others)
    {
        int owner = -1;
        for (size_t k = 0; k < chain.size(); k++)
            if (i > chain[k].pack && i < chain[k].unpack)
                owner = (int)k;
        if (owner < 0)
            return fail(layers[i].type() + " " + layers[i].name() + " lies outside every Pack..Unpack chain");
        int& slot = layers[i].type() == "SeedVR2MMRoPE" ? chain[owner].rope : chain[owner].attention;
        if (slot >= 0)
            return fail("two " + layers[i].type() + " layers in the chain of " + layers[chain[owner].pack].name());
        slot = i;
    }

    for (size_t k = 0; k < chain.size(); k++)
    {
        ChainLayers& c = chain[k];
        const Layer& pack = layers[c.pack];
        const Layer& unpack = layers[c.unpack];
        auto wired = [&](int consumer, const std::string& blob) {
            return layers[consumer].bottom(0) == blob;
        };
        if (c.rope >= 0 && !wired(c.rope, pack.top(0)))
            return fail("SeedVR2MMRoPE " + layers[c.rope].name() + " does not read " + pack.name() + "'s packed output " +
                        pack.top(0));
        if (c.rope >= 0 && c.attention >= 0 && !wired(c.attention, layers[c.rope].top(0)))
            return fail("SeedVR2WindowAttention " + layers[c.attention].name() + " does not read " +
                        layers[c.rope].name() + "'s output " + layers[c.rope].top(0));
        if (c.attention >= 0 && !wired(c.unpack, layers[c.attention].top(0)))
            return fail("SeedVR2AWAUnpack " + unpack.name() + " does not read " + layers[c.attention].name() +
                        "'s output " + layers[c.attention].top(0));
        if (c.rope < 0 && c.attention < 0 && wired(c.unpack, pack.top(0)))
            return fail("SeedVR2AWAUnpack " + unpack.name() + " reads the packed rows with no attention between");
        const int members[4] = {c.pack, c.rope, c.attention, c.unpack};
        for (int m : members)
        {
            if (m < 0)
                continue;
            for (int id = 0; id < 8; id++)
                if (params[m].value[id] != params[c.pack].value[id] &&
                    !(id == 7 && (params[m].value[7] != 0) == (params[c.pack].value[7] != 0)))
                    return fail(layers[m].name() + " disagrees with " + pack.name() + " on parameter " +
                                std::to_string(id));
        }
        const bool dynamic = params[c.pack].value[0] == -1;
        const long long video_tokens = dynamic ? -1 : params[c.pack].value[0] * params[c.pack].value[1] *
                                                          params[c.pack].value[2];
        int reshape_height = 0;
        for (size_t i = 0; i < layers.size(); i++)
        {
            const Layer& layer = layers[i];
            if (layer.type() != "Reshape" || layer.bottoms != 1 || layer.tops != 1 ||
                layer.bottom(0) != unpack.top(0) || layer.name().compare(0, 23, "reshape_awa_video_batch") != 0)
                continue;
            if (c.reshape >= 0)
                return fail("two video batch reshapes read " + unpack.name() + "'s video output");
            c.reshape = (int)i;
            int found = 0;
            long long height = 0;
            for (size_t f = layer.param_start; f < layer.fields.size(); f++)
                if (layer.fields[f].compare(0, 2, "1=") == 0)
                {
                    found++;
                    if (!parse_int(layer.fields[f].substr(2), height))
                        found = 2;
                }
            if (found != 1)
                return fail(layer.name() + " must have exactly one integer height parameter");
            if (height != video_tokens)
                return fail(layer.name() + " height " + std::to_string(height) + " does not match the " +
                            (dynamic ? std::string("dynamic grid (-1)") :
                                       std::to_string(video_tokens) + " video tokens of the grid"));
            reshape_height = (int)height;
        }
        if ((int)k < capacity && chains)
        {
            awa_graph_chain& out = chains[k];
            std::memset(&out, 0, sizeof(out));
            const long long* v = params[c.pack].value;
            out.params.source_t = (int)v[0];
            out.params.source_h = (int)v[1];
            out.params.source_w = (int)v[2];
            out.params.windows_t = (int)v[3];
            out.params.windows_h = (int)v[4];
            out.params.windows_w = (int)v[5];
            out.params.text_tokens = (int)v[6];
            out.params.shifted = v[7] != 0 ? 1 : 0;
            out.params.rope_dim = c.rope >= 0 && params[c.rope].present[8] ? (int)params[c.rope].value[8] : 126;
            out.dynamic = dynamic ? 1 : 0;
            out.pack_line = layers[c.pack].line_number;
            out.rope_line = c.rope >= 0 ? layers[c.rope].line_number : 0;
            out.attention_line = c.attention >= 0 ? layers[c.attention].line_number : 0;
            out.unpack_line = layers[c.unpack].line_number;
            out.reshape_line = c.reshape >= 0 ? layers[c.reshape].line_number : 0;
            out.reshape_height = reshape_height;
        }
    }
    return (int)chain.size();
}

bool read_file(const char* path, std::string& data, std::string& error)
{
    std::ifstream input(path, std::ios::binary);
    if (!input)
    {
        error = std::string("cannot open ") + path;
        return false;
    }
    data.assign(std::istreambuf_iterator<char>(input), std::istreambuf_iterator<char>());
    if (input.bad())
    {
        error = std::string("cannot read ") + path;
        return false;
    }
    return true;
}

// ---------------------------------------------------------------- manifest
// The package check of the reference's model registry
// (src/model/model_registry.cpp:248-362), built here as three steps: read the
// manifest into records, list the package's files with a walker of its own,
// compare the two. The rules and the messages are the registry's (a package
// must be accepted or refused the same way by both runtimes); the code is not.
struct ManifestRecord
{
    std::string name;
    std::string digest;  // lowercase hex
};

// A manifest path: relative, POSIX separators, no empty ("//"), "." or ".."
// component and no backslash (the registry's safe_manifest_path, as
// std::filesystem reads a path on POSIX: a single trailing '/' is allowed).
bool manifest_path_ok(const std::string& name)
{
    if (name.empty() || name[0] == '/' || name.find('\\') != std::string::npos ||
        name.find("//") != std::string::npos)
        return false;
    size_t begin = 0;
    while (begin <= name.size())
    {
        size_t end = name.find('/', begin);
        if (end == std::string::npos)
            end = name.size();
        const std::string part = name.substr(begin, end - begin);
        if (part == "." || part == "..")
            return false;
        begin = end + 1;
    }
    return true;
}

int hex_value(char c)
{
    if (c >= '0' && c <= '9')
        return c - '0';
    if (c >= 'a' && c <= 'f')
        return c - 'a' + 10;
    if (c >= 'A' && c <= 'F')
        return c - 'A' + 10;
    return -1;
}

// Reads manifest.sha256 into records sorted by name. A record line is 64 hex
// digits, two spaces and a path; CR line ends and blank lines are allowed.
bool read_manifest(const std::filesystem::path& file, std::vector<ManifestRecord>& records, std::string& error)
{
    std::string text;
    {
        std::ifstream input(file, std::ios::binary);
        if (!input)
        {
            error = "missing model package manifest: " + file.string();
            return false;
        }
        text.assign(std::istreambuf_iterator<char>(input), std::istreambuf_iterator<char>());
    }
    std::set<std::string> names;
    size_t number = 0, pos = 0;
    while (pos < text.size())
    {
        size_t stop = text.find('\n', pos);
        if (stop == std::string::npos)
            stop = text.size();
        std::string line = text.substr(pos, stop - pos);
        pos = stop + 1;
        ++number;
        if (!line.empty() && line.back() == '\r')
            line.pop_back();
        if (line.empty())
            continue;
        ManifestRecord rec;
        bool hex = line.size() > 66 && line.compare(64, 2, "  ") == 0 && line.find("  ") == 64;
        for (size_t i = 0; hex && i < 64; i++)
        {
            const int v = hex_value(line[i]);
            hex = v >= 0;
            rec.digest.push_back("0123456789abcdef"[v < 0 ? 0 : v]);
        }
        if (!hex)
        {
            error = "invalid model package manifest record at line " + std::to_string(number);
            return false;
        }
        rec.name = line.substr(66);
        if (!manifest_path_ok(rec.name))
        {
            error = "invalid model package manifest path at line " + std::to_string(number);
            return false;
        }
        if (!names.insert(rec.name).second)
        {
            error = "duplicate model package manifest path: " + rec.name;
            return false;
        }
        records.push_back(std::move(rec));
    }
    std::sort(records.begin(), records.end(),
              [](const ManifestRecord& a, const ManifestRecord& b) { return a.name < b.name; });
    return true;
}

// Every regular file under dir (except the top-level manifest) as
// (relative POSIX name, path), sorted by name. Directories are entered, never
// followed through links; any link is refused.
bool list_package(const std::filesystem::path& dir, std::vector<std::pair<std::string, std::filesystem::path>>& files,
                  std::string& error)
{
    namespace fs = std::filesystem;
    const std::string inspect = "failed to inspect model package: " + dir.string();
    std::vector<fs::path> pending{dir};
    while (!pending.empty())
    {
        const fs::path here = pending.back();
        pending.pop_back();
        std::error_code ec;
        fs::directory_iterator it(here, ec), end;
        if (ec)
        {
            error = inspect;
            return false;
        }
        for (; it != end; it.increment(ec))
        {
            if (ec)
            {
                error = inspect;
                return false;
            }
            const fs::file_status st = it->symlink_status(ec);
            if (ec)
            {
                error = inspect;
                return false;
            }
            if (fs::is_symlink(st))
            {
                error = "model package must not contain symbolic links: " + it->path().string();
                return false;
            }
            if (fs::is_directory(st))
                pending.push_back(it->path());
            else if (fs::is_regular_file(st))
            {
                std::string name = it->path().lexically_relative(dir).generic_string();
                if (name != "manifest.sha256")
                    files.emplace_back(std::move(name), it->path());
            }
        }
        if (ec)
        {
            error = inspect;
            return false;
        }
    }
    std::sort(files.begin(), files.end());
    for (size_t i = 1; i < files.size(); i++)
        if (files[i].first == files[i - 1].first)
        {
            error = "duplicate model package artifact path: " + files[i].first;
            return false;
        }
    return true;
}

// expected_records: 0 = the registry's rule (75 records for a positive-only
// package, 146 with the CFG branch), > 0 = exactly that many, < 0 = any.
bool validate_manifest(const std::filesystem::path& dir, int expected_records, std::string& error)
{
    std::vector<ManifestRecord> records;
    if (!read_manifest(dir / "manifest.sha256", records, error))
        return false;
    const size_t count = records.size();
    if (expected_records == 0 && count != 75 && count != 146)
    {
        error = "model package manifest must contain 75 records (positive) or 146 records (positive + CFG), got " +
                std::to_string(count);
        return false;
    }
    if (expected_records > 0 && count != (size_t)expected_records)
    {
        error = "model package manifest must contain " + std::to_string(expected_records) + " records, got " +
                std::to_string(count);
        return false;
    }
    std::vector<std::pair<std::string, std::filesystem::path>> files;
    if (!list_package(dir, files, error))
        return false;
    auto by_name = [](const std::pair<std::string, std::filesystem::path>& f, const std::string& n) {
        return f.first < n;
    };
    // every record names a file whose digest it holds (records in name order) ...
    for (const ManifestRecord& rec : records)
    {
        const auto hit = std::lower_bound(files.begin(), files.end(), rec.name, by_name);
        if (hit == files.end() || hit->first != rec.name)
        {
            error = "manifest artifact is missing: " + rec.name;
            return false;
        }
        std::string digest;
        if (!sha256_file(hit->second, digest, error))
            return false;
        if (digest != rec.digest)
        {
            error = "manifest hash mismatch for artifact: " + rec.name;
            return false;
        }
    }
    // ... and no file is left out (files in name order)
    if (files.size() != records.size())
        for (const auto& f : files)
        {
            const auto hit = std::lower_bound(records.begin(), records.end(), f.first,
                                              [](const ManifestRecord& r, const std::string& n) { return r.name < n; });
            if (hit == records.end() || hit->name != f.first)
            {
                error = "artifact is not listed in model package manifest: " + f.second.string();
                return false;
            }
        }
    return true;
}

}  // namespace

extern "C" {

int awa_graph_find_chains(const char* param_text, size_t length, awa_graph_chain* chains, int capacity)
{
    if (!param_text && length)
        return fail("awa_graph_find_chains: null text");
    if (capacity < 0 || (capacity > 0 && !chains))
        return fail("awa_graph_find_chains: invalid chain buffer");
    try
    {
        return find_chains(param_text ? param_text : "", length, chains, capacity);
    }
    catch (const std::exception& e)
    {
        return report_error(AWA_ERR_ALLOC, e.what());
    }
}

int awa_graph_find_chains_file(const char* param_path, awa_graph_chain* chains, int capacity)
{
    if (!param_path)
        return fail("awa_graph_find_chains_file: null path");
    try
    {
        std::string data, error;
        if (!read_file(param_path, data, error))
            return fail(error);
        return awa_graph_find_chains(data.data(), data.size(), chains, capacity);
    }
    catch (const std::exception& e)
    {
        return report_error(AWA_ERR_ALLOC, e.what());
    }
}

int awa_graph_make_dynamic(const char* param_text, size_t length, char* out, size_t capacity, size_t* out_length)
{
    if ((!param_text && length) || !out_length || (capacity && !out))
        return fail("awa_graph_make_dynamic: invalid arguments");
    try
    {
        std::string result, error;
        if (!make_dynamic(param_text ? param_text : "", length, result, error))
            return fail(error);
        *out_length = result.size();
        if (capacity < result.size())
            return report_error(AWA_ERR_ALLOC, "awa_graph_make_dynamic: output buffer too small");
        std::memcpy(out, result.data(), result.size());
        if (capacity > result.size())
            out[result.size()] = '\0';
        return AWA_OK;
    }
    catch (const std::exception& e)
    {
        return report_error(AWA_ERR_ALLOC, e.what());
    }
}

int awa_manifest_validate(const char* package_dir, int expected_records)
{
    if (!package_dir)
        return fail("awa_manifest_validate: null directory");
    try
    {
        std::string error;
        if (!validate_manifest(std::filesystem::path(package_dir), expected_records, error))
            return fail(error);
        return AWA_OK;
    }
    catch (const std::exception& e)
    {
        return fail(std::string("failed to inspect model package: ") + e.what());
    }
}

int awa_sha256(const void* data, size_t size, char* hex)
{
    if (!hex || (!data && size))
        return fail("awa_sha256: invalid arguments");
    Sha256 hash;
    hash.update(static_cast<const unsigned char*>(data), size);
    const std::string digest = hash.hex();
    std::memcpy(hex, digest.c_str(), 65);
    return AWA_OK;
}

int awa_sha256_file(const char* path, char* hex)
{
    if (!path || !hex)
        return fail("awa_sha256_file: invalid arguments");
    try
    {
        std::string digest, error;
        if (!sha256_file(std::filesystem::path(path), digest, error))
            return fail(error);
        std::memcpy(hex, digest.c_str(), 65);
        return AWA_OK;
    }
    catch (const std::exception& e)
    {
        return fail(e.what());
    }
}

}  // extern "C"
