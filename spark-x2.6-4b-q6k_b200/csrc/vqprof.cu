// vqprof.cu — VQPROF 1 tuning profiles: the artifact fingerprint, the reader with its trust
// rules, the writer. Host code only.
//
// A profile names, per matrix geometry, the kernel measured fastest for it on one device
// (tools/vq/gpu/vq-profile.h:1-40, the format; tools/vq-tune/src/profile.rs, the writer).
// It is advisory, as in the reference runtime (vq-model-gpu.cu:1094-1122): a caller applies
// it only when it parsed with version 1, was tuned on the same artifact (the fingerprint
// below) and names this device; spk_model_use_profile then replaces the kernel heuristic per
// geometry where the named kernel can run (vq-model-gpu.cu:301-324).
//
// The fingerprint (vq-profile.h:19-26): FNV-1a 64 over the manifest.txt bytes as stored, then,
// for every matrix line of the manifest in file order whose stage count is above zero, the
// matrix name, its container's size as 8 little-endian bytes, and the container's first and
// last min(4096, size) bytes (a container of at most 4096 bytes contributes its bytes twice).
// A matrix line is `name rows cols stages bytes relL2`, all six fields present (lines that
// start with '#' and empty lines are skipped), as the runtime's reader takes them
// (vq-profile.h:122-131).
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "common.cuh"
#include "spk.h"

using spk::set_error;

namespace {

// FNV-1a with the 64-bit prime; the starting value is the one both sides of the format use
// (vq-profile.h:66, vq-tune/src/artifact.rs:14), 1469598103934665603, which is not the
// published 64-bit offset basis: a fingerprint has to start from it to match theirs.
constexpr uint64_t FNV_OFFSET = 1469598103934665603ull;
constexpr uint64_t FNV_PRIME = 1099511628211ull;

uint64_t fnv1a(uint64_t h, const unsigned char *p, size_t n) {
    for (size_t i = 0; i < n; i++) {
        h ^= p[i];
        h *= FNV_PRIME;
    }
    return h;
}

bool read_file(const std::string &path, std::vector<unsigned char> &out) {
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    out.clear();
    unsigned char buf[1 << 16];
    size_t n;
    while ((n = fread(buf, 1, sizeof buf, f)) > 0) out.insert(out.end(), buf, buf + n);
    const bool ok = !ferror(f);
    fclose(f);
    return ok;
}

// One container: name, size (8 bytes LE), first and last edge.
bool hash_container(uint64_t &h, const std::string &dir, const std::string &name) {
    const std::string path = dir + "/" + name + ".bin";
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    bool ok = fseek(f, 0, SEEK_END) == 0;
    const long sz = ok ? ftell(f) : -1;
    ok = ok && sz >= 0 && fseek(f, 0, SEEK_SET) == 0;
    if (!ok) {
        fclose(f);
        return false;
    }
    const uint64_t size = (uint64_t)sz;
    h = fnv1a(h, (const unsigned char *)name.data(), name.size());
    unsigned char le[8];
    for (int i = 0; i < 8; i++) le[i] = (unsigned char)(size >> (8 * i));
    h = fnv1a(h, le, 8);
    const size_t edge = size < 4096 ? (size_t)size : 4096;
    std::vector<unsigned char> head(edge), tail(edge);
    ok = fread(head.data(), 1, edge, f) == edge;
    if (ok && size > 4096) ok = fseek(f, (long)(size - 4096), SEEK_SET) == 0 && fread(tail.data(), 1, 4096, f) == 4096;
    else tail = head;
    fclose(f);
    if (!ok) return false;
    h = fnv1a(h, head.data(), edge);
    h = fnv1a(h, tail.data(), edge);
    return true;
}

// The trailing newline, carriage return and spaces of a line go (vq-profile.h:144-148).
void trim_end(std::string &s) {
    while (!s.empty() && (s.back() == '\n' || s.back() == '\r' || s.back() == ' ')) s.pop_back();
}

bool starts(const std::string &s, const char *p) { return s.compare(0, strlen(p), p) == 0; }

}  // namespace

extern "C" {

int spk_vqprof_fingerprint(const char *dir, unsigned long long *out) {
    if (!dir || !out) return set_error("vqprof fingerprint: dir and out are required");
    const std::string d(dir);
    std::vector<unsigned char> man;
    if (!read_file(d + "/manifest.txt", man)) return set_error("%s/manifest.txt cannot be read", dir);
    uint64_t h = fnv1a(FNV_OFFSET, man.data(), man.size());
    size_t p = 0;
    while (p < man.size()) {
        size_t e = p;
        while (e < man.size() && man[e] != '\n') e++;
        const std::string line(man.begin() + p, man.begin() + e);
        if (!line.empty() && line[0] != '#') {
            char name[1024];
            unsigned long long rows, cols, stages, bytes;
            double rel;
            if (sscanf(line.c_str(), "%1023s %llu %llu %llu %llu %lf", name, &rows, &cols, &stages, &bytes, &rel) == 6 &&
                stages > 0 && !hash_container(h, d, name))
                return set_error("%s/%s.bin, listed in the manifest, cannot be read", dir, name);
        }
        p = e + 1;
    }
    *out = h;
    return 0;
}

int spk_vqprof_load(const char *path, spk_vqprof *pf) {
    if (!path || !pf) return set_error("vqprof load: path and profile are required");
    memset(pf, 0, sizeof *pf);
    FILE *f = fopen(path, "r");
    if (!f) return set_error("profile %s cannot be opened", path);
    char buf[512];
    while (fgets(buf, sizeof buf, f)) {
        std::string line(buf);
        trim_end(line);
        if (starts(line, "VQPROF ")) {
            pf->version = atoi(line.c_str() + 7);
            continue;
        }
        if (starts(line, "artifact ")) {
            unsigned long long v = 0;
            if (sscanf(line.c_str() + 9, "%llx", &v) == 1) pf->artifact = v;
            continue;
        }
        if (starts(line, "gpu ")) {
            snprintf(pf->gpu, sizeof pf->gpu, "%s", line.c_str() + 4);
            continue;
        }
        if (starts(line, "driver ")) {
            snprintf(pf->driver, sizeof pf->driver, "%s", line.c_str() + 7);
            continue;
        }
        spk_vqprof_entry e;
        memset(&e, 0, sizeof e);
        double rate = 0.0;
        int n = sscanf(line.c_str(), "gemv %d %d %d %d %d %d %d %lf", &e.dim, &e.nc, &e.rows, &e.cols, &e.v3, &e.variant,
                       &e.threads, &rate);
        if (n >= 7) {
            e.kind = 0;
        } else if ((n = sscanf(line.c_str(), "prefill %d %d %d %d %d %d %d %d %lf", &e.dim, &e.nc, &e.rows, &e.cols,
                               &e.v3, &e.variant, &e.bn, &e.bk, &rate)) >= 8) {
            e.kind = 1;
        } else {
            continue;   // an unknown directive: skipped, as the runtime's reader does
        }
        e.rate = rate;
        if (pf->n < SPK_VQPROF_MAX) pf->e[pf->n++] = e;
    }
    fclose(f);
    if (pf->version != SPK_VQPROF_VERSION)
        return set_error("profile %s is version %d, not %d", path, pf->version, SPK_VQPROF_VERSION);
    return 0;
}

int spk_vqprof_find(const spk_vqprof *pf, int kind, int dim, int nc, int rows, int cols, int v3) {
    if (!pf) return -1;
    for (int i = 0; i < pf->n && i < SPK_VQPROF_MAX; i++) {
        const spk_vqprof_entry &e = pf->e[i];
        if (e.kind == kind && e.dim == dim && e.nc == nc && e.rows == rows && e.cols == cols && e.v3 == v3) return i;
    }
    return -1;
}

int spk_vqprof_trust(const spk_vqprof *pf, unsigned long long artifact, const char *device) {
    if (!pf || !device) return set_error("vqprof trust: profile and device are required");
    if (pf->version != SPK_VQPROF_VERSION) return 3;
    if (pf->artifact != artifact) return 1;
    if (strcmp(pf->gpu, device) != 0) return 2;
    return 0;
}

int spk_vqprof_write(const char *path, const spk_vqprof *pf) {
    if (!path || !pf) return set_error("vqprof write: path and profile are required");
    if (pf->n < 0 || pf->n > SPK_VQPROF_MAX) return set_error("vqprof write: %d entries (0..%d)", pf->n, SPK_VQPROF_MAX);
    std::string s = "VQPROF " + std::to_string(SPK_VQPROF_VERSION) + "\n";
    char line[512];
    snprintf(line, sizeof line, "artifact %016llx\ngpu %s\ndriver %s\n", pf->artifact, pf->gpu, pf->driver);
    s += line;
    for (int i = 0; i < pf->n; i++) {
        const spk_vqprof_entry &e = pf->e[i];
        if (e.kind == 0)
            snprintf(line, sizeof line, "gemv %d %d %d %d %d %d %d %.1f\n", e.dim, e.nc, e.rows, e.cols, e.v3 ? 1 : 0,
                     e.variant, e.threads, e.rate);
        else
            snprintf(line, sizeof line, "prefill %d %d %d %d %d %d %d %d %.1f\n", e.dim, e.nc, e.rows, e.cols,
                     e.v3 ? 1 : 0, e.variant, e.bn, e.bk, e.rate);
        s += line;
    }
    // through a temporary file and a rename: a reader never sees half a profile
    const std::string tmp = std::string(path) + ".tmp";
    FILE *f = fopen(tmp.c_str(), "wb");
    if (!f) return set_error("%s cannot be written", tmp.c_str());
    const bool ok = fwrite(s.data(), 1, s.size(), f) == s.size();
    if (fclose(f) != 0 || !ok) {
        remove(tmp.c_str());
        return set_error("%s: short write", tmp.c_str());
    }
    if (rename(tmp.c_str(), path) != 0) {
        remove(tmp.c_str());
        return set_error("%s cannot be renamed to %s", tmp.c_str(), path);
    }
    return 0;
}

}  // extern "C"
