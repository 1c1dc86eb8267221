// st_harness.cpp -- runs the reference's own safetensors parser
// (model/safetensors.cpp, compiled unmodified from the reference tree by
// `make st REF=...`) on one file and prints what it accepted, as JSON.
//
// Test infrastructure: tests/golden/make_st_golden.py runs it on the cases of
// tests/st_cases.py and commits the output (tests/golden/st_cases.json), so the
// parity tests never need the reference tree. argv[2] selects the options:
// "strict" (the checkpoint loader's, weight_index.cpp:20-27) or "loose"
// (no dtype, header or data alignment requirement).
#include <cstdio>
#include <string>

#include "model/safetensors.h"

static std::string esc(const std::string& s) {
    std::string o;
    for (char c : s) {
        if (c == '"' || c == '\\') o += '\\';
        if (static_cast<unsigned char>(c) < 0x20) {
            char b[8];
            std::snprintf(b, sizeof b, "\\u%04x", c);
            o += b;
            continue;
        }
        o += c;
    }
    return o;
}

int main(int argc, char** argv) {
    if (argc < 3) return 2;
    glm::SafeTensorsOptions o;
    if (std::string(argv[2]) == "strict") {
        o.requireBf16 = true;
        o.requireAlignedHeader = true;
        o.requireAlignedData = true;
        o.allowF32NameContaining.push_back("e_score_correction_bias");
    } else {
        o.requireBf16 = false;
        o.requireAlignedHeader = false;
        o.requireAlignedData = false;
    }
    glm::SafeTensorsFile f;
    const bool ok = f.open(argv[1], o);
    const glm::SafeTensorsStats& s = f.validationStats();
    std::printf("{\"ok\": %s, \"stats\": {\"total\": %zu, \"accepted\": %zu, \"rejected\": %zu, "
                "\"duplicate_rejected\": %zu, \"dtype_rejected\": %zu, "
                "\"f32_allowed_accepted\": %zu, \"shape_rejected\": %zu, "
                "\"bounds_rejected\": %zu, \"byte_mismatch_rejected\": %zu, "
                "\"alignment_rejected\": %zu}, \"tensors\": [",
                ok ? "true" : "false", s.total, s.accepted, s.rejected, s.duplicateRejected,
                s.dtypeRejected, s.f32AllowedAccepted, s.shapeRejected, s.boundsRejected,
                s.byteMismatchRejected, s.alignmentRejected);
    bool first = true;
    if (ok) {
        for (const auto& kv : f.tensors()) {
            const glm::TensorInfo& t = kv.second;
            std::printf("%s{\"name\": \"%s\", \"dtype\": \"%s\", \"shape\": [", first ? "" : ", ",
                        esc(t.name).c_str(), esc(t.dtype).c_str());
            for (size_t d = 0; d < t.shape.size(); ++d)
                std::printf("%s%d", d ? ", " : "", t.shape[d]);
            std::printf("], \"offset\": %llu, \"bytes\": %llu}",
                        (unsigned long long)(f.headerSize() + t.dataBegin),
                        (unsigned long long)t.byteSize());
            first = false;
        }
    }
    std::printf("]}\n");
    return 0;
}
