#!/usr/bin/env bash
# Run one configuration on the GPUs of this node under torchrun (one process per GPU,
# rendezvous on 127.0.0.1): prepare, train and predict, logging to a file.
#
#   examples/run_multi_gpu.sh CONFIG [NUM_GPUS] [PHASE] [extra CLI flags...]
#   examples/run_multi_gpu.sh configs/mpnn_lstm_nvlink.yaml 4
#   examples/run_multi_gpu.sh configs/tgn_large_nvlink.yaml 8 train --epochs 3
#
# PHASE is all (default), prepare, train or predict. Environment: PORT (rendezvous port,
# default 29500), LOG_DIR (default ./logs), WALL_S (hard bound on the torchrun call, default
# 86400 s; the process group's own dist.timeout_s bounds each collective well below it).
set -euo pipefail

CONFIG="${1:?usage: $0 CONFIG [NUM_GPUS] [PHASE] [extra flags]}"
NGPU="${2:-$(nvidia-smi -L 2>/dev/null | wc -l)}"
PHASE="${3:-all}"
shift $(( $# < 3 ? $# : 3 ))
PORT="${PORT:-29500}"
LOG_DIR="${LOG_DIR:-./logs}"
WALL_S="${WALL_S:-86400}"
ROOT="$(cd "$(dirname "${BASH_SOURCE[0]}")/.." && pwd)"
mkdir -p "${LOG_DIR}"
LOG="${LOG_DIR}/$(basename "${CONFIG}" .yaml)_${NGPU}gpu_$(date +%Y%m%d_%H%M%S).log"
export PYTHONPATH="${ROOT}${PYTHONPATH:+:${PYTHONPATH}}"

log() { echo "[$(date '+%H:%M:%S')] $*" | tee -a "${LOG}"; }

if [[ "${NGPU}" -lt 1 ]]; then
    echo "no GPU found (pass NUM_GPUS explicitly)" >&2
    exit 2
fi
log "config=${CONFIG} gpus=${NGPU} phase=${PHASE} log=${LOG}"
# one torchrun call for every phase: rank 0 writes the artifacts while the others wait, and one
# process group serves prepare, train and predict
timeout -k 60 "${WALL_S}" python -m torch.distributed.run --nnodes=1 --nproc-per-node "${NGPU}" \
    --master-addr 127.0.0.1 --master-port "${PORT}" \
    -m starry_unigraph --config "${CONFIG}" --phase "${PHASE}" "$@" 2>&1 | tee -a "${LOG}"
log "done"
