"""Track 1 on B200: DUST with ANVIL II on the block matrices and Adam elsewhere, without backpropagation.

The entry point of train/val/run.py with the work in noise_b200: same command line (:659-668), recipe
and overrides (:41-73, :679-686), data shuffle (:688-689), warmup-then-rebuild (:708-713), linear
warmdown (:702-706) and outputs (config.json, metrics.jsonl, final.pt, result.json; :690-746). The
estimator (capture, direct reruns, coordinate head, local attention reruns, reassembly, mixing-scalar
ES) and the optimizers run on the sm_100a kernels behind noise_b200's C ABI. FineWeb rows are read from
--data-dir when present; --synthetic substitutes seeded Zipf(1.1) rows of the same shape.

Launch: torchrun --standalone --nproc_per_node=8 train/val/run.py [--synthetic]
"""
import argparse
from dataclasses import asdict
import datetime
import json
import os
from pathlib import Path
import sys
import time

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from noise_b200.data import ROW, TRAIN_ROWS, VAL_ROWS, load_rows  # noqa: E402
from noise_b200.dust import DUST, recipe  # noqa: E402
from noise_b200.model import Weights  # noqa: E402
from noise_b200.optim import make_optimizer  # noqa: E402
from noise_b200.population import evaluate  # noqa: E402

BATCH = 8  # sequences per update; 610 updates per epoch
SEED = 0


def main(track: str = 'val', default_scale: float = 1.0, target: float | None = None):
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--data-dir', type=Path, default=Path('data'))
    parser.add_argument('--output', type=Path, default=Path(f'logs/{track}'))
    parser.add_argument('--scale', type=float, help='Scale every draw count of the 16k Adam cell instead.')
    parser.add_argument('--warmdown', type=float, help='Override the recipe\'s warmdown fraction.')
    parser.add_argument('--lr', type=float, help='Override the recipe\'s Adam learning rate.')
    parser.add_argument('--anvil-lr', type=float, help='Override the recipe\'s ANVIL II learning rate.')
    parser.add_argument('--steps', type=int, help='Stop after this many updates (smoke tests).')
    parser.add_argument('--eval-every', type=int, default=0, help='Untimed validation every this many updates.')
    parser.add_argument('--synthetic', action='store_true', help='Zipf(1.1) rows when the FineWeb files are absent.')
    args = parser.parse_args()

    if not torch.cuda.is_available():
        parser.error('Training requires a CUDA GPU.')
    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group('nccl', device_id=device, timeout=datetime.timedelta(minutes=20))
    settings = recipe(args.scale if args.scale else default_scale)
    if args.warmdown is not None:
        settings.warmdown = args.warmdown
    if args.lr is not None:
        settings.lr = args.lr
    if args.anvil_lr is not None:
        settings.anvil_lr = args.anvil_lr

    training = load_rows(args.data_dir / 'train.pt', TRAIN_ROWS, args.synthetic, seed=1)
    training = training[torch.randperm(len(training), generator=torch.Generator().manual_seed(SEED + 1))]
    steps = min(len(training) // BATCH, args.steps or len(training))
    if rank == 0:
        if args.output.exists() and any(args.output.iterdir()):
            raise FileExistsError(f'Choose an empty output directory: {args.output}')
        args.output.mkdir(parents=True, exist_ok=True)
        config = dict(script=f'train/{track}/run.py', world=world, batch=BATCH, steps=steps, seed=SEED)
        if target is not None:
            config['target'] = target
        config.update(recipe=asdict(settings), torch_version=torch.__version__, backend='noise_b200 sm_100a')
        (args.output / 'config.json').write_text(json.dumps(config, indent=2) + '\n')

    def init():
        model = Weights(device, seed=SEED)
        optimizer = make_optimizer(model, settings.lr, settings.betas, settings.anvil_lr, settings.anvil_wd, steps)
        return model, optimizer, DUST(model, settings, SEED, rank, world)

    def set_rate(optimizer, step):
        left = (steps - step + 1) / steps
        for group in optimizer.param_groups:
            group.setdefault('initial_lr', group['lr'])
            group['lr'] = group['initial_lr'] * min(1.0, left / settings.warmdown if settings.warmdown else 1.0)

    # untimed warmup on random tokens, then rebuild from the seed
    model, optimizer, estimator = init()
    noise = torch.randint(0, 4096, (BATCH, ROW), generator=torch.Generator().manual_seed(SEED)).to(device)
    estimator.step(noise[:, :-1].contiguous(), noise[:, 1:].contiguous(), optimizer)
    model, optimizer, estimator = init()
    val = load_rows(args.data_dir / 'val.pt', VAL_ROWS, args.synthetic, seed=2)

    if rank == 0:
        print(f'{track}: {steps} steps, recipe={asdict(settings)}, GPUs={world}', flush=True)
    log = (args.output / 'metrics.jsonl').open('a') if rank == 0 else None
    torch.cuda.synchronize()
    start, paused, elapsed = time.perf_counter(), 0.0, 0.0
    step = 0
    for step in range(1, steps + 1):
        batch = training[(step - 1) * BATCH:step * BATCH].to(device)
        set_rate(optimizer, step)
        loss = estimator.step(batch[:, :-1].contiguous(), batch[:, 1:].contiguous(), optimizer)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - start - paused
        record = dict(step=step, train_loss=loss, train_seconds=round(elapsed, 2))
        if args.eval_every and step % args.eval_every == 0 and step < steps:
            pause = time.perf_counter()
            record['val_loss'] = evaluate(model, val)
            paused += time.perf_counter() - pause
        if rank == 0:
            print(json.dumps(record), flush=True)
            log.write(json.dumps(record) + '\n')
            log.flush()

    state = model.state_dict()
    val_loss = evaluate(model, val)
    if rank == 0:
        torch.save(state, args.output / 'final.pt')
        result = dict(val_loss=val_loss, train_seconds=round(elapsed, 2), steps=step, tokens=step * BATCH * 2048)
        if target is not None:
            result['reached_target'] = val_loss <= target
        (args.output / 'result.json').write_text(json.dumps(result, indent=2) + '\n')
        print(json.dumps(result), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == '__main__':
    main()
