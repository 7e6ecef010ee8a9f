#!/usr/bin/env bash
# Test infrastructure only. Builds the UNMODIFIED reference gten library
# (iangitonga/nanochatllms.cpp) straight from the reference checkout, together with
# oracle/ref_harness.cpp, into oracle/_ref/libgtenref.so.
#
# Flags follow the reference build (CMakeLists.txt:10-12,64,117: -O3 -mavx -mf16c), plus:
#   -fopenmp        : the reference's CMake FindOpenMP does not detect OpenMP with this
#                     toolchain, so it is passed explicitly (the matmul loop ops.cpp:601-603).
#   -include cstring: minicpm/minicpm.cpp:24 uses std::memcpy without including <cstring>.
# Nothing is copied out of the reference tree; outputs go to oracle/_ref/ only.
set -euo pipefail
HERE="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
# The checkout: the first argument, else $GTEN_REFERENCE_DIR, else BASELINE.json's reference_path.
REF="${1:-${GTEN_REFERENCE_DIR:-}}"
if [ -z "$REF" ]; then
    REF="$(python3 -c 'import json,sys; print(json.load(open(sys.argv[1])).get("reference_path") or "")' \
           "$HERE/../BASELINE.json" 2>/dev/null || true)"
fi
OUT="$HERE/_ref"
if [ -z "$REF" ] || [ ! -d "$REF/src/gten" ]; then
    echo "reference checkout not found at $REF; keeping any prebuilt $OUT/libgtenref.so" >&2
    exit 0
fi
mkdir -p "$OUT/obj"
CXX="${CXX:-g++}"
FLAGS="-O3 -mavx -mf16c -std=c++17 -fopenmp -fPIC -include cstring -w -I$REF/src"
SRCS=(
  "$REF/src/gten/ops.cpp"
  "$REF/src/gten/quants.cpp"
  "$REF/src/gten/tensor.cpp"
  "$REF/src/gten/utils.cpp"
  "$REF/src/gten/modules.cpp"
  "$REF/src/tinyllama/tinyllama.cpp"
  "$REF/src/zephyr/zephyr.cpp"
  "$REF/src/minicpm/minicpm.cpp"
  "$REF/src/openelm/openelm.cpp"
  "$REF/src/gten/tokenizer.cpp"
  "$HERE/ref_harness.cpp"
  "$HERE/tok_harness.cpp"
)
OBJS=()
pids=()
for s in "${SRCS[@]}"; do
    o="$OUT/obj/$(basename "$(dirname "$s")")_$(basename "${s%.cpp}").o"
    OBJS+=("$o")
    if [ ! -f "$o" ] || [ "$s" -nt "$o" ]; then
        $CXX $FLAGS -c "$s" -o "$o" &
        pids+=($!)
    fi
done
for p in "${pids[@]}"; do wait "$p"; done
# Link the OpenMP runtime by path: this toolchain's driver does not find libgomp.spec.
GOMP="$($CXX -print-file-name=libgomp.so.1)"
[ -f "$GOMP" ] || GOMP=/usr/lib/x86_64-linux-gnu/libgomp.so.1
# Link the shared libstdc++ by path too: where the driver only finds libstdc++.a, the library would
# carry its own copy, whose locale facets (GNU-unique symbols) clash with the shared copy that
# other modules of the same process load (std::regex in Gpt2Tokenizer then crashes).
STDCXX="$($CXX -print-file-name=libstdc++.so.6)"
[ -f "$STDCXX" ] || STDCXX=/usr/lib/x86_64-linux-gnu/libstdc++.so.6
$CXX -shared -o "$OUT/libgtenref.so" "${OBJS[@]}" "$STDCXX" "$GOMP" -lpthread
echo "built $OUT/libgtenref.so"
