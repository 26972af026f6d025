"""Launch helpers: the Slurm/torchrun launcher (``train.slurm`` beside this file)
and ``python -m avgen_b200.launch.preflight`` (scripts/train.slurm and
scripts/preflight.sh roles in the reference)."""
