#!/usr/bin/env bash
# Runs the framework's checks tier by tier and stops at the first failure.
#
#   ./run_checks.sh          CPU tiers: algebra and unit tests, then the Gloo tier
#   ./run_checks.sh --gpu    also the CUDA tier (a B200 with the extension built in-tree)
#
# The Gloo tier needs permission to bind local sockets; where that is refused
# the script fails instead of reporting a skipped tier as a pass. Reference
# parity tests need the reference package under baseline/_ref (or the
# directory in NMB_REFERENCE_PATH) and skip without it; the script says so.
set -euo pipefail
cd "$(dirname "$0")"

PYTHON=${PYTHON:-python3}
GPU=0
for arg in "$@"; do
    case "$arg" in
        --gpu) GPU=1 ;;
        -h|--help) sed -n '2,10p' "$0"; exit 0 ;;
        *) echo "unknown argument: $arg" >&2; exit 2 ;;
    esac
done

ref_dir=${NMB_REFERENCE_PATH:-baseline/_ref}
if [[ -d "$ref_dir/nano_megatron" ]]; then
    echo "reference package: $ref_dir (parity tests run)"
else
    echo "reference package: not found under $ref_dir (parity tests skip)"
fi

echo
echo "== algebra, units, protocol model checks (no sockets) =="
$PYTHON -m pytest -q -m "not gpu and not distributed"

echo
echo "== Gloo processes: collectives, matrix vs the unsharded model, CLI, failures =="
if ! $PYTHON - <<'PY' 2>/dev/null
import socket
s = socket.socket()
s.bind(("127.0.0.1", 0))
s.close()
PY
then
    echo "FAIL: binding a local socket is not permitted here; Gloo cannot run," >&2
    echo "so the distributed tier was not checked." >&2
    exit 1
fi
$PYTHON -m pytest -q -m "distributed and not gpu"
$PYTHON -m tests.test_parallel_matrix --matrix

if [[ $GPU == 1 ]]; then
    echo
    echo "== CUDA: kernels vs fp32 torch, model vs CPU, fused collectives on every visible GPU =="
    $PYTHON -c "import torch, sys; sys.exit(0 if torch.cuda.is_available() else 'no CUDA device visible')"
    $PYTHON -c "import nano_megatron_b200.ops.cuda"  # fails with the build command if the extension is missing
    $PYTHON -m pytest -q -m gpu
fi
echo
echo "all checks passed"
