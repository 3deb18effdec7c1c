#!/usr/bin/env bash
# Compile the reference runtime (Fovane/Sabah-MoE-Accelerator
# sabah/runtime/cuda/sabah_rt.cu) from its sources where they lie, unmodified,
# into oracle/_ref/libsabah_rt_ref.so. Test infrastructure: the tests use its
# sabah_rt_host_dequant to pin the oracle and its sabah_rt_mul_mat_id_v2 /
# sabah_moe_block as the reference GPU path; bench.py --impl reference times its
# host dequantizer as the reference CPU path.
#
# The source is Windows-first. Three defines make it build on Linux without
# editing it: <string> is included up front, HANDLE/INVALID_HANDLE_VALUE get
# stand-ins, and `lanes` (a member that exists only in the Win32 struct, read
# once at sabah_rt.cu:1318) is mapped to the Linux member `fd`, which is -1 for
# every unopened file, so that guarded branch is inert exactly as lanes == 0 is.
set -euo pipefail
HERE="$(cd "$(dirname "$0")" && pwd)"
# the reference project: SABAH_REF_ROOT, else beside this repository
REF_ROOT="${SABAH_REF_ROOT:-$HERE/../../reference}"
SRC="$REF_ROOT/sabah/runtime/cuda/sabah_rt.cu"
OUT="$HERE/_ref"
if [ ! -f "$SRC" ]; then
    echo "reference source not found: $SRC" >&2
    exit 2
fi
mkdir -p "$OUT"
nvcc -O3 -gencode arch=compute_100a,code=sm_100a -shared -Xcompiler -fPIC \
    -include string -DHANDLE='void*' -DINVALID_HANDLE_VALUE='((void*)-1)' -Dlanes=fd \
    -diag-suppress 550,177 \
    "$SRC" -o "$OUT/libsabah_rt_ref.so"
echo "built $OUT/libsabah_rt_ref.so"
