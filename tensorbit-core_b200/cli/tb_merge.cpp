/// @file tb_merge.cpp
/// @brief tb-merge: native counterpart of the reference's scripts/merge_tbm.py.
///
///   tb-merge --input ./pruned/shard1/ ./pruned/shard2/ --output ./pruned/full/model.tbm
///            [--architecture llama]
///
/// Same flags, output bytes, messages (stdout) and exit codes as the script
/// (merge_tbm.py:158-213): 0 on success, 1 when no valid .tb file was found or
/// a file could not be read or written, 2 for a command-line error.  Long
/// options may be abbreviated and written as --opt=value, as argparse allows.

#include <cstdio>
#include <string>
#include <string_view>
#include <vector>

#include "tensorbit/core/merge.hpp"

namespace {

constexpr const char* kUsage =
    "usage: tb-merge [-h] --input INPUT [INPUT ...] --output OUTPUT [--architecture ARCHITECTURE]\n";

int usage_error(const std::string& msg) {
    std::fputs(kUsage, stderr);
    std::fprintf(stderr, "tb-merge: error: %s\n", msg.c_str());
    return 2;
}

/// The long option `arg` names (exact, or an unambiguous prefix), or "".
std::string match_option(std::string_view arg) {
    static const char* kOpts[] = {"--input", "--output", "--architecture", "--help"};
    std::string hit;
    for (const char* o : kOpts) {
        const std::string_view opt(o);
        if (opt == arg) return std::string(opt);
        if (arg.size() > 2 && opt.substr(0, arg.size()) == arg) {
            if (!hit.empty()) return "?";
            hit = opt;
        }
    }
    return hit;
}

}  // namespace

int main(int argc, char** argv) {
    std::vector<std::string> inputs;
    std::string output, architecture = "llama";
    bool have_input = false, have_output = false;
    for (int i = 1; i < argc; ++i) {
        std::string arg = argv[i];
        std::string value;
        bool inline_value = false;
        if (arg.rfind("--", 0) == 0) {
            const auto eq = arg.find('=');
            if (eq != std::string::npos) {
                value = arg.substr(eq + 1);
                arg.resize(eq);
                inline_value = true;
            }
        }
        const std::string opt = arg == "-h" ? "--help" : match_option(arg);
        if (opt == "?") return usage_error("ambiguous option: " + arg);
        if (opt == "--help") {
            std::fputs(kUsage, stdout);
            std::puts("\nMerge .tb directories into a unified .tbm container");
            return 0;
        }
        if (opt.empty()) return usage_error("unrecognized arguments: " + arg);
        auto take_one = [&](std::string& dst) -> bool {
            if (inline_value) { dst = value; return true; }
            if (i + 1 >= argc || (argv[i + 1][0] == '-' && argv[i + 1][1] != '\0')) return false;
            dst = argv[++i];
            return true;
        };
        if (opt == "--input") {
            inputs.clear();
            if (inline_value) {
                inputs.push_back(value);
            } else {
                while (i + 1 < argc && !(argv[i + 1][0] == '-' && argv[i + 1][1] != '\0')) inputs.emplace_back(argv[++i]);
            }
            if (inputs.empty()) return usage_error("argument --input: expected at least one argument");
            have_input = true;
        } else if (opt == "--output") {
            if (!take_one(output)) return usage_error("argument --output: expected one argument");
            have_output = true;
        } else if (opt == "--architecture") {
            if (!take_one(architecture)) return usage_error("argument --architecture: expected one argument");
        }
    }
    if (!have_input || !have_output) {
        std::string missing;
        if (!have_input) missing = "--input";
        if (!have_output) missing += missing.empty() ? "--output" : ", --output";
        return usage_error("the following arguments are required: " + missing);
    }

    tensorbit::core::MergeReport report;
    const auto r = tensorbit::core::merge_tb_directories(inputs, output, architecture, &report);
    for (const auto& line : report.log) std::puts(line.c_str());
    if (!r.has_value()) {
        if (r.error() != tensorbit::core::MergeError::kNoInputs) std::fprintf(stderr, "tb-merge: %s\n", report.detail.c_str());
        return 1;
    }
    return 0;
}
