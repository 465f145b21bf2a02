#!/bin/sh
# Test infrastructure: builds the reference's own `realdataset_search` CUDA binary
# for sm_100a, used only as the same-run parity and speed comparison on the GPU box.
#
# Usage: oracle/build_ref.sh <reference-checkout> [<out-dir>]
#
# The reference sources are copied to a scratch directory outside the repository and
# two edits are applied to that copy only (they are the edits the reference's own main
# needs for a 2-attribute 4x4 grid):
#   1. realdataset_search.cu main(): attr_dim 1 -> 2 and shape {16} -> {4,4}
#      (the attribute count and grid shape are compile-time constants there).
#   2. realdataset_search.cu: the loop that overwrites the ranges of queries >= 992
#      with those of query i-10 is made empty (start index set to query_num).
# Nothing from the reference tree is written into the repository; the binary goes to
# <out-dir> (default oracle/_ref), which is git-ignored.
set -eu
REF="$1"
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="${2:-$HERE/_ref}"
SCRATCH=$(mktemp -d /tmp/gf_refbuild.XXXXXX)
cp -r "$REF/indexsearch" "$SCRATCH/"
SRC="$SCRATCH/indexsearch/realdataset_search.cu"
grep -q 'for(unsigned i = 992 ; i < query_num ; i ++) {' "$SRC"
sed -i 's/for(unsigned i = 992 ; i < query_num ; i ++) {/for(unsigned i = query_num ; i < query_num ; i ++) {/' "$SRC"
sed -i '/^int main(int argc , char\*\* argv) {$/,/string attrD/{s/constexpr unsigned attr_dim = 1 ;/constexpr unsigned attr_dim = 2 ;/;s/vector<unsigned> shape = {16} ;/vector<unsigned> shape = {4 , 4} ;/}' "$SRC"
grep -q 'constexpr unsigned attr_dim = 2 ;' "$SRC"
grep -q 'vector<unsigned> shape = {4 , 4} ;' "$SRC"
mkdir -p "$OUT"
cd "$SCRATCH/indexsearch"
nvcc -O3 -o "$OUT/realdataset_search" realdataset_search.cu \
    -gencode arch=compute_100a,code=sm_100a -Xcompiler -fopenmp --extended-lambda -w \
    -Xcompiler -mcmodel=medium -Xlinker --no-relax -lcublas
echo "built $OUT/realdataset_search"
