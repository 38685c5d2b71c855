#!/usr/bin/env bash
# Builds the reference arm of bench.py into baseline/_ref (git-ignored; it travels to the GPU box with
# the rest of the tree). Steps: copy the read-only reference tree to a scratch directory, run the
# reference's own build-time patch step (scripts/apply_ggml_vm_c.sh, idempotent), then configure and
# build its vendored ggml (CUDA + CPU backends) and libllama with the reference's ggml options plus the
# driver in this directory. Architecture: sm_100 SASS only ("100-real"; the reference's own GPU query
# picks "100", which adds compute_100 PTX that a B200 never JIT-compiles since the SASS matches). Offline: the only third-party header libllama needs (nlohmann/json, for
# its jinja engine) is taken from a copy bundled with an installed Python package.
#
#   baseline/build_ref.sh [REFERENCE_TREE] [JOBS]
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
SRC_IN="${1:-/root/reference}"
JOBS="${2:-$(nproc)}"
OUT="${HERE}/_ref"
SCRATCH="${OUT}/src"
mkdir -p "${OUT}"
rm -rf "${SCRATCH}"
cp -r "${SRC_IN}" "${SCRATCH}"
chmod -R u+w "${SCRATCH}"
bash "${SCRATCH}/scripts/apply_ggml_vm_c.sh"
JSON_DIR="$(python3 - <<'PY'
import glob, os, site
for base in site.getsitepackages():
    for p in glob.glob(os.path.join(base, "**", "nlohmann", "json.hpp"), recursive=True):
        print(os.path.dirname(os.path.dirname(p)))
        raise SystemExit
PY
)"
test -n "${JSON_DIR}" || { echo "nlohmann/json.hpp not found" >&2; exit 1; }
cmake -S "${HERE}" -B "${OUT}/build" -G Ninja -DCMAKE_BUILD_TYPE=Release \
  -DCMAKE_CUDA_ARCHITECTURES=100-real -DVMC_REF_SRC="${SCRATCH}" -DVMC_JSON_INCLUDE="${JSON_DIR}"
cmake --build "${OUT}/build" --target vmc_ref_bench -j "${JOBS}"
cp "${OUT}/build/vmc_ref_bench" "${OUT}/vmc_ref_bench"
# CPU-only stack (vendored libllama + ggml-cpu): the config-1 oracle; runs without a GPU driver.
cmake -S "${HERE}" -B "${OUT}/build_cpu" -G Ninja -DCMAKE_BUILD_TYPE=Release -DVMC_REF_CUDA=OFF \
  -DVMC_REF_SRC="${SCRATCH}" -DVMC_JSON_INCLUDE="${JSON_DIR}"
cmake --build "${OUT}/build_cpu" --target vmc_ref_bench -j "${JOBS}"
cp "${OUT}/build_cpu/vmc_ref_bench" "${OUT}/vmc_ref_cpu"
echo "built ${OUT}/vmc_ref_bench and ${OUT}/vmc_ref_cpu"
