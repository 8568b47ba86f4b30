#!/usr/bin/env bash
# Captures rung summaries from the runners that oracle/runner_build.sh builds,
# as fixtures for the summary-schema tests (tests/test_summary_schema.py).
# Needs a B200. Usage: tests/golden/capture_runner_summaries.sh OUT_DIR
# The device UUID and PCI bus id are replaced by placeholders; every other
# field is the runner's own output.
set -euo pipefail
REPO="$(cd "$(dirname "$0")/../.." && pwd)"
OUT="${1:?output directory}"
mkdir -p "$OUT"
G="$REPO/oracle/_ref/gpu-power-runner-gplk"
R="$REPO/oracle/_ref/gpu-power-runner"
COMMON=(--warmup-sec 1 --steady-sec 2 --sample-hz 50)

rung() {  # rung NAME BINARY ARGS...
  local name="$1" bin="$2"; shift 2
  local tmp="$OUT/$name.raw.json"
  local rc=0
  "$bin" "${COMMON[@]}" --out-summary "$tmp" "$@" > /dev/null 2>&1 || rc=$?
  python3 - "$tmp" "$OUT/$name.json" <<'EOF'
import json, sys
doc = json.load(open(sys.argv[1]))
doc["device"]["uuid"] = "GPU-00000000-0000-0000-0000-000000000000"
doc["device"]["pci_bus_id"] = "00000000:00:00.0"
json.dump(doc, open(sys.argv[2], "w"), indent=1, sort_keys=False)
EOF
  rm -f "$tmp"
  echo "$name rc=$rc"
}

rung gplk_memstream "$G" --op memstream --size 32768
rung gplk_sgemm_fp32 "$G" --op sgemm --precision fp32 --size 1024
rung gplk_sgemm_fp8 "$G" --op sgemm --precision fp8 --size 8192
rung gplk_sgemm_fp4 "$G" --op sgemm --precision fp4 --size 8192
rung gplk_powervirus "$G" --op powervirus --size 4096 --duty-on-ms 100 --duty-off-ms 100
if [ -x "$R" ]; then
  rung ref_memstream "$R" --op memstream --size 32768
  rung ref_sgemm_fp32 "$R" --op sgemm --precision fp32 --size 1024
  rung ref_sgemm_fp4_rejected "$R" --op sgemm --precision fp4 --size 4096
  rung ref_powervirus "$R" --op powervirus --size 4096 --duty-on-ms 100 --duty-off-ms 100
  rung ref_powervirus_capped "$R" --op powervirus --size 8192 --tensor-backend cublas --precision bf16 --mix-fma 0 --mix-dram 0
fi
