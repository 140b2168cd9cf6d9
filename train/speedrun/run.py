"""Track 2 on B200: the shortest training time to reach validation loss TARGET, without backpropagation.

The track 1 estimator and optimizers (train/val/run.py) at the reference's 5k population,
recipe(0.3125) (train/speedrun/run.py:41, :76); result.json adds reached_target.

Launch: torchrun --standalone --nproc_per_node=8 train/speedrun/run.py [--synthetic]
"""
from pathlib import Path
import sys

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from train.val.run import main  # noqa: E402

TARGET = 4.2  # validation loss to reach; the run counts only if its final weights reach it

if __name__ == '__main__':
    main(track='speedrun', default_scale=0.3125, target=TARGET)
