// Minimal stand-in for absl logging used ONLY to compile reference sources
// as test oracles (oracle/build_ref.py): LOG / VLOG write to stderr.
#pragma once
#include <iostream>

#define LOG(severity) std::cerr << "[" #severity "] "
#define VLOG(level) if (false) std::cerr
