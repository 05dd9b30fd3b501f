"""Generate videos with a PAN 2 checkpoint: ``python generate.py --prompt "..." --checkpoint_path ...``;
``torchrun --nproc-per-node 8 generate.py --sp_size 8 ...`` for sequence-parallel sampling.
Options: ``python generate.py --help``."""
from pan2_b200.generate import main

if __name__ == "__main__":
    main()
