"""Train the PAN 2 MMDiT: ``torchrun --nproc-per-node 8 train.py --config config/pretrain_29B_720p.yaml``.

Options are the reference trainer's (YAML keys = option names, the command line overrides the YAML);
see ``python train.py --help``.
"""
from pan2_b200.training.trainer import main

if __name__ == "__main__":
    main()
