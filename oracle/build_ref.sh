#!/bin/sh
# Test infrastructure: builds the reference's own `realdataset_search` CUDA binary
# for sm_100a, used only as the same-run parity and speed comparison on the GPU box.
#
# Usage: oracle/build_ref.sh <reference-checkout> [<out-dir>]
#
# The reference sources are copied to a scratch directory outside the repository and
# four edits are applied to that copy only:
#   1. realdataset_search.cu main(): attr_dim 1 -> 2 and shape {16} -> {4,4}
#      (the attribute count and grid shape are compile-time constants there).
#   2. realdataset_search.cu: the loop that overwrites the ranges of queries >= 992
#      with those of query i-10 is made empty (start index set to query_num).
#   3. real_dataset_adapter.cuh: prefiltering_tag_elements is launched with the
#      2 * attr_dim * sizeof(T) bytes of dynamic shared memory its body writes the
#      query box into (the shipped launch passes none, which is an out-of-bounds
#      shared-memory write for every query: an illegal memory access on B200).
#   4. real_dataset_adapter.cuh: the bool array indices_is_little_seg (selected_num
#      bytes) is allocated 4 * qnum bytes longer and zeroed, because the planner's
#      sort_by_clustering_info_weighted reads it as unsigned[qnum] (its p_ls_counts
#      argument); with fewer than 4 selected cells per query that read ends past the
#      allocation.  Zero there means "no exact-route cells", what the reference means
#      with --prefilter 0.
# Edits 3 and 4 change no result the reference computes on valid memory.  Nothing
# from the reference tree is written into the repository; the binary goes to
# <out-dir> (default oracle/_ref), which is git-ignored.
set -eu
REF="$1"
HERE=$(cd "$(dirname "$0")" && pwd)
OUT="${2:-$HERE/_ref}"
SCRATCH=$(mktemp -d /tmp/gf_refbuild.XXXXXX)
cp -r "$REF/indexsearch" "$SCRATCH/"
SRC="$SCRATCH/indexsearch/realdataset_search.cu"
ADA="$SCRATCH/indexsearch/real_dataset_adapter.cuh"
grep -q 'for(unsigned i = 992 ; i < query_num ; i ++) {' "$SRC"
sed -i 's/for(unsigned i = 992 ; i < query_num ; i ++) {/for(unsigned i = query_num ; i < query_num ; i ++) {/' "$SRC"
sed -i '/^int main(int argc , char\*\* argv) {$/,/string attrD/{s/constexpr unsigned attr_dim = 1 ;/constexpr unsigned attr_dim = 2 ;/;s/vector<unsigned> shape = {16} ;/vector<unsigned> shape = {4 , 4} ;/}' "$SRC"
grep -q 'constexpr unsigned attr_dim = 2 ;' "$SRC"
grep -q 'vector<unsigned> shape = {4 , 4} ;' "$SRC"
sed -i 's/prefiltering_tag_elements<T><<<qnum , 32>>>(/prefiltering_tag_elements<T><<<qnum , 32 , 2 * attr_dim * sizeof(T)>>>(/' "$ADA"
grep -q 'prefiltering_tag_elements<T><<<qnum , 32 , 2 \* attr_dim \* sizeof(T)>>>(' "$ADA"
sed -i 's/cudaMalloc((void\*\*) &indices_is_little_seg , selected_num \* sizeof(bool)) ;/cudaMalloc((void**) \&indices_is_little_seg , (selected_num + 4 * qnum) * sizeof(bool)) ; cudaMemset(indices_is_little_seg , 0 , (selected_num + 4 * qnum) * sizeof(bool)) ;/' "$ADA"
test "$(grep -c 'cudaMemset(indices_is_little_seg , 0 , (selected_num + 4 \* qnum) \* sizeof(bool))' "$ADA")" -eq 2
mkdir -p "$OUT"
cd "$SCRATCH/indexsearch"
nvcc -O3 -o "$OUT/realdataset_search" realdataset_search.cu \
    -gencode arch=compute_100a,code=sm_100a -Xcompiler -fopenmp --extended-lambda -w \
    -Xcompiler -mcmodel=medium -Xlinker --no-relax -lcublas
echo "built $OUT/realdataset_search"
