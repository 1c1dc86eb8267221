// host_fuzz.cpp -- the library's host-side code on hostile and random input,
// built with AddressSanitizer and UndefinedBehaviorSanitizer (no GPU needed).
//
// Checkpoint shards are untrusted input: hf_st_open parses a JSON header whose
// length, offsets and shapes come from the file. This program takes every
// file of a seed corpus (the parser cases of tests/st_cases.py, written by
// tests/test_sanitizers_cpu.py), opens each one and many seeded mutations of
// it (bytes flipped or set to JSON punctuation, truncations, spans repeated,
// the 8-byte header length rewritten) with the strict and the loose options,
// and walks every accepted tensor: hf_st_tensor, hf_st_find, hf_st_read into
// a buffer of exactly the reported size (and one byte short, which must
// fail). It also feeds hf_st_layer_shards mutated checkpoint indexes and the
// expert-parallel planners random loads and counts, checking the invariants
// their callers rely on (a placement is a permutation with E/W experts per
// rank; an exchange plan places every received row exactly once) and context
// creation random configurations (refused on the host, never a crash).
//
// Usage: host_fuzz <corpus dir> <scratch dir> <iterations> <seed>
// Exit 0 when every check held; a sanitizer report aborts the program.
#include <dirent.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <random>
#include <string>
#include <vector>

#include "hf_ingest.h"
#include "hf_moe.h"

static int g_failures = 0;
static long g_opened = 0, g_tensors = 0;  // files opened, accepted tensors walked

#define CHECK(cond, ...)                                        \
    do {                                                        \
        if (!(cond)) {                                          \
            std::fprintf(stderr, "CHECK failed: %s: ", #cond); \
            std::fprintf(stderr, __VA_ARGS__);                  \
            std::fprintf(stderr, "\n");                         \
            ++g_failures;                                       \
        }                                                       \
    } while (0)

static std::vector<unsigned char> read_file(const std::string& p) {
    std::ifstream f(p, std::ios::binary);
    return std::vector<unsigned char>((std::istreambuf_iterator<char>(f)),
                                      std::istreambuf_iterator<char>());
}

static void write_file(const std::string& p, const std::vector<unsigned char>& b) {
    std::ofstream f(p, std::ios::binary | std::ios::trunc);
    f.write(reinterpret_cast<const char*>(b.data()), std::streamsize(b.size()));
}

// Opens `path` with one set of options and exercises every accepted tensor.
static void walk(const std::string& path, bool strict) {
    static const char* allow[] = {"e_score_correction_bias"};
    hf_st_options strict_o{1, allow, 1, 1, 1};
    hf_st_options loose_o{0, nullptr, 0, 0, 0};
    hf_st_file* f = nullptr;
    hf_st_stats st{};
    if (hf_st_open(path.c_str(), strict ? &strict_o : &loose_o, &f, &st) != HF_OK) {
        CHECK(f == nullptr, "a failed open returned a file");
        return;
    }
    ++g_opened;
    const int n = hf_st_count(f);
    g_tensors += n;
    CHECK(n >= 0 && uint64_t(n) == st.accepted, "count %d vs accepted %llu", n,
          (unsigned long long)st.accepted);
    CHECK(st.accepted + st.rejected == st.total, "accepted + rejected != total");
    for (int i = 0; i < n; ++i) {
        const char *name = nullptr, *dtype = nullptr;
        int ndim = 0;
        int64_t shape[8];
        uint64_t off = 0, bytes = 0;
        if (hf_st_tensor(f, i, &name, &dtype, &ndim, shape, 8, &off, &bytes) != HF_OK) {
            CHECK(false, "hf_st_tensor failed on accepted tensor %d", i);
            continue;
        }
        CHECK(name && dtype && ndim > 0 && bytes > 0, "tensor %d incomplete", i);
        // a name given twice keeps its last entry, so find() returns some index with that name
        const int j = name ? hf_st_find(f, name) : -1;
        CHECK(j >= 0 && j < n, "find(%s) = %d", name ? name : "?", j);
        if (bytes > (uint64_t(64) << 20)) continue;  // span checked against the file size already
        std::vector<unsigned char> buf(size_t(bytes) + 1);
        CHECK(hf_st_read(f, i, buf.data(), bytes) == HF_OK, "read of tensor %d", i);
        CHECK(hf_st_read(f, i, buf.data(), bytes - 1) == HF_ERR_ARG, "short buffer accepted");
    }
    CHECK(hf_st_find(f, "no.such.tensor") == -1, "find of a missing name");
    CHECK(hf_st_tensor(f, n, nullptr, nullptr, nullptr, nullptr, 0, nullptr, nullptr) != HF_OK,
          "tensor past the end");
    hf_st_close(f);
}

static std::vector<unsigned char> mutate(std::vector<unsigned char> b, std::mt19937_64& rng) {
    static const char punct[] = "{}[]\":,0123456789-.eE\\u \t\n";
    const int rounds = 1 + int(rng() % 4);
    for (int r = 0; r < rounds; ++r) {
        const size_t n = b.size();
        switch (rng() % 7) {
            case 0:  // flip a bit
                if (n) b[rng() % n] ^= static_cast<unsigned char>(1u << (rng() % 8));
                break;
            case 1:  // a byte becomes JSON punctuation or a digit
                if (n) b[rng() % n] = static_cast<unsigned char>(punct[rng() % (sizeof(punct) - 1)]);
                break;
            case 2:  // truncate
                if (n) b.resize(rng() % n);
                break;
            case 3: {  // repeat a span
                if (n < 2) break;
                const size_t a = rng() % n, len = 1 + rng() % std::min<size_t>(64, n - a);
                std::vector<unsigned char> span(b.begin() + long(a), b.begin() + long(a + len));
                const size_t at = rng() % n;
                b.insert(b.begin() + long(at), span.begin(), span.end());
                break;
            }
            case 4: {  // rewrite the header length near its value, or anywhere
                if (n < 8) break;
                uint64_t h = 0;
                std::memcpy(&h, b.data(), 8);
                const uint64_t v = (rng() % 4 == 0) ? rng() : h + (rng() % 33) - 16;
                std::memcpy(b.data(), &v, 8);
                break;
            }
            case 5:  // a digit inside the header becomes a large number
                for (int tries = 0; tries < 16 && n > 9; ++tries) {
                    const size_t p = 8 + rng() % (n - 8);
                    if (b[p] >= '0' && b[p] <= '9') {
                        const char* big[] = {"4294967296", "18446744073709551615",
                                             "99999999999999999999", "1e30", "-1", "1073741825"};
                        const std::string s = big[rng() % 6];
                        b.erase(b.begin() + long(p));
                        b.insert(b.begin() + long(p), s.begin(), s.end());
                        break;
                    }
                }
                break;
            default:  // append junk
                for (int i = 0, m = int(rng() % 16); i < m; ++i)
                    b.push_back(static_cast<unsigned char>(rng()));
                break;
        }
    }
    return b;
}

static void fuzz_layer_shards(const std::string& dir, std::mt19937_64& rng, int iters) {
    write_file(dir + "/model-00001-of-00002.safetensors", {});
    write_file(dir + "/model-00002-of-00002.safetensors", {});
    const std::string base =
        "{\"metadata\": {\"total_size\": 1}, \"weight_map\": {"
        "\"model.layers.3.mlp.gate.weight\": \"model-00002-of-00002.safetensors\", "
        "\"model.layers.3.mlp.experts.0.up_proj.weight\": \"model-00001-of-00002.safetensors\"}}";
    std::vector<unsigned char> seed(base.begin(), base.end());
    std::vector<char> buf(1 << 16);
    for (int it = 0; it < iters; ++it) {
        std::vector<unsigned char> idx = it == 0 ? seed : mutate(seed, rng);
        write_file(dir + "/model.safetensors.index.json", idx);
        int n = -1;
        const hf_status s = hf_st_layer_shards(dir.c_str(), 3, buf.data(), buf.size(), &n);
        if (it == 0) CHECK(s == HF_OK && n == 2, "seed index: status %d, %d shards", int(s), n);
        if (s == HF_OK) {
            CHECK(n >= 0 && n <= 2, "%d shards from a 2-shard directory", n);
            size_t pos = 0;
            for (int i = 0; i < n; ++i) {
                const size_t len = std::strlen(buf.data() + pos);
                CHECK(len > 0 && pos + len < buf.size(), "shard path %d", i);
                pos += len + 1;
            }
        }
    }
    std::remove((dir + "/model.safetensors.index.json").c_str());
    std::remove((dir + "/model-00001-of-00002.safetensors").c_str());
    std::remove((dir + "/model-00002-of-00002.safetensors").c_str());
}

static void fuzz_planners(std::mt19937_64& rng, int iters) {
    for (int it = 0; it < iters; ++it) {
        const int W = 1 << int(rng() % 4);           // 1, 2, 4, 8
        const int E = W * (1 + int(rng() % 32));
        std::vector<long long> load(static_cast<size_t>(E));
        for (auto& l : load) l = (rng() % 3 == 0) ? 0 : (long long)(rng() % 100000);
        std::vector<int32_t> order(static_cast<size_t>(E), -1);
        CHECK(hf_ep_balanced_placement(E, W, load.data(), order.data()) == HF_OK, "placement");
        std::vector<int32_t> sorted = order;
        std::sort(sorted.begin(), sorted.end());
        for (int e = 0; e < E; ++e) CHECK(sorted[size_t(e)] == e, "placement is not a permutation");
        for (int r = 0; r < W; ++r)
            CHECK(std::is_sorted(order.begin() + long(r) * (E / W),
                                 order.begin() + long(r + 1) * (E / W)),
                  "rank %d's experts not ascending", r);

        const int El = 1 + int(rng() % 8), T = int(rng() % 64), has_shared = int(rng() % 2);
        std::vector<int32_t> send(size_t(W) * El), recv(size_t(W) * El);
        for (auto& v : send) v = int32_t(rng() % 20);
        for (auto& v : recv) v = int32_t(rng() % 20);
        int R = 0;
        for (int v : recv) R += v;
        std::vector<int32_t> soff(size_t(W) + 1), roff(size_t(W) + 1), lc(size_t(El) + 1);
        std::vector<int32_t> rows(size_t(R + T) + 1, -1), rpos(size_t(R) + 1, -1);
        CHECK(hf_ep_plan(W, El, T, has_shared, send.data(), recv.data(), soff.data(), roff.data(),
                         lc.data(), rows.data(), rpos.data()) == HF_OK, "plan");
        CHECK(roff[size_t(W)] == R, "recv_off total %d vs %d", roff[size_t(W)], R);
        std::vector<int> seen(size_t(R), 0);
        for (int p = 0; p < R; ++p) {
            const int row = rows[size_t(p)];
            CHECK(row >= 0 && row < R, "position %d -> row %d", p, row);
            if (row >= 0 && row < R) {
                ++seen[size_t(row)];
                CHECK(rpos[size_t(row)] == p, "row_pos does not invert local_rows");
            }
        }
        for (int r = 0; r < R; ++r) CHECK(seen[size_t(r)] == 1, "row %d placed %d times", r, seen[size_t(r)]);
        if (has_shared)
            for (int t = 0; t < T; ++t) CHECK(rows[size_t(R + t)] == R + t, "shared row %d", t);
    }
}

// Context creation validates its configuration on the host before touching a
// device: on a machine without a GPU every config below is refused with
// HF_ERR_ARG or, when it is valid, HF_ERR_UNSUPPORTED (never a crash). Skipped
// where a device exists (valid configs would allocate for real).
static void fuzz_configs(std::mt19937_64& rng, int iters) {
    hf_moe_config probe{64, 8, 2, 32, 32, 2.5f, 1, 1, 4, 0, 0, 0, 0, 1, nullptr};
    hf_moe_ctx* pc = nullptr;
    if (hf_moe_create(&pc, &probe) == HF_OK) {
        hf_moe_destroy(pc);
        return;
    }
    const int pick[] = {-1, 0, 1, 7, 8, 9, 64, 255, 256, 1024, 1025, 6144, 1 << 30, 2147483647};
    for (int it = 0; it < iters; ++it) {
        auto r = [&] { return pick[rng() % (sizeof(pick) / sizeof(pick[0]))]; };
        hf_moe_config c{};
        c.hidden_size = r();
        c.num_experts = r();
        c.num_experts_per_tok = r();
        c.moe_intermediate_size = r();
        c.shared_intermediate_size = r();
        c.routed_scaling_factor = 2.5f;
        c.norm_topk_prob = 1;
        c.num_layers = r();
        c.max_tokens = r();
        c.device = int(rng() % 3) - 1;
        c.path = int(rng() % 5) - 1;
        c.gemv_max_tokens = r();
        c.ep_world = 1;
        hf_moe_ctx* ctx = nullptr;
        const hf_status s = hf_moe_create(&ctx, &c);
        CHECK(s == HF_ERR_ARG || s == HF_ERR_UNSUPPORTED, "create returned %d", int(s));
        CHECK(ctx == nullptr, "a failed create returned a context");
        const size_t w = hf_dense_mlp_workspace_size(r(), r(), r());
        (void)w;
    }
}

int main(int argc, char** argv) {
    if (argc != 5) {
        std::fprintf(stderr, "usage: %s <corpus dir> <scratch dir> <iterations> <seed>\n", argv[0]);
        return 2;
    }
    const std::string corpus = argv[1], scratch = argv[2];
    const int iters = std::atoi(argv[3]);
    std::mt19937_64 rng(std::strtoull(argv[4], nullptr, 10));
    std::vector<std::vector<unsigned char>> seeds;
    if (DIR* d = opendir(corpus.c_str())) {
        std::vector<std::string> names;
        while (dirent* e = readdir(d)) {
            const std::string n = e->d_name;
            if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) names.push_back(n);
        }
        closedir(d);
        std::sort(names.begin(), names.end());
        for (const std::string& n : names) {
            const std::string p = corpus + "/" + n;
            walk(p, true);
            walk(p, false);
            seeds.push_back(read_file(p));
        }
    }
    CHECK(!seeds.empty(), "no seed files in %s", corpus.c_str());
    if (seeds.empty()) return 1;
    const std::string tmp = scratch + "/mutant.safetensors";
    // headers nested far deeper than any checkpoint (the reader must not
    // recurse without bound) and a header length past the file
    for (const std::string& h : {std::string(200000, '['), [] {
             std::string s;
             for (int i = 0; i < 100000; ++i) s += "{\"a\":";
             return s;
         }()}) {
        std::vector<unsigned char> b(8);
        const uint64_t len = h.size();
        std::memcpy(b.data(), &len, 8);
        b.insert(b.end(), h.begin(), h.end());
        b.resize(b.size() + 64, ' ');
        write_file(tmp, b);
        walk(tmp, true);
        walk(tmp, false);
        const uint64_t past = len + 1000;
        std::memcpy(b.data(), &past, 8);
        write_file(tmp, b);
        walk(tmp, false);
    }
    for (int it = 0; it < iters; ++it) {
        write_file(tmp, mutate(seeds[rng() % seeds.size()], rng));
        walk(tmp, (it & 1) == 0);
    }
    std::remove(tmp.c_str());
    fuzz_layer_shards(scratch, rng, iters / 10 + 1);
    fuzz_planners(rng, iters / 10 + 1);
    fuzz_configs(rng, iters / 10 + 1);
    std::printf("%s: %d seeds, %d mutants, %ld opens accepted, %ld tensors walked, %d failed checks\n",
                g_failures ? "FAIL" : "OK", int(seeds.size()), iters, g_opened, g_tensors, g_failures);
    return g_failures ? 1 : 0;
}
