#include "core/env.h"

#include <cstdlib>
#include <cstring>
#include <sstream>

namespace bccl {

long EnvInt(const char* name, long dflt) {
    const char* v = std::getenv(name);
    if (v == nullptr || *v == '\0') return dflt;
    char* end = nullptr;
    long r = std::strtol(v, &end, 0);
    if (end == v) return dflt;
    // Accept K/M/G suffixes for sizes.
    if (end && (*end == 'k' || *end == 'K')) r <<= 10;
    if (end && (*end == 'm' || *end == 'M')) r <<= 20;
    if (end && (*end == 'g' || *end == 'G')) r <<= 30;
    return r;
}

std::string EnvStr(const char* name, const std::string& dflt) {
    const char* v = std::getenv(name);
    return (v == nullptr || *v == '\0') ? dflt : std::string(v);
}

bool EnvFlag(const char* name) {
    const char* v = std::getenv(name);
    if (v == nullptr) return false;
    return !strcmp(v, "1") || !strcasecmp(v, "true") || !strcasecmp(v, "yes") || !strcasecmp(v, "on");
}

bool FaultActive(const char* site, int rank, long* arg) {
    const char* v = std::getenv("BCCL_FAULT");
    if (v == nullptr || *v == '\0') return false;
    std::stringstream ss(v);
    std::string item;
    while (std::getline(ss, item, ',')) {
        std::stringstream is(item);
        std::string s, r, a;
        std::getline(is, s, ':');
        std::getline(is, r, ':');
        std::getline(is, a, ':');
        if (s != site) continue;
        if (!r.empty() && r != "*" && std::atoi(r.c_str()) != rank) continue;
        if (arg) *arg = a.empty() ? 0 : std::atol(a.c_str());
        return true;
    }
    return false;
}

}  // namespace bccl
