#!/bin/sh
# Builds the CPU oracle (test infrastructure): an AVX2 and an AVX-512 variant.
set -e
cd "$(dirname "$0")"
g++ -O3 -mavx2 -mfma -fopenmp -fPIC -shared -std=c++17 -o liboracle_avx2.so osor_oracle.cpp
g++ -O3 -mavx512f -mavx512vl -mavx2 -mfma -fopenmp -fPIC -shared -std=c++17 -o liboracle_avx512.so osor_oracle.cpp
