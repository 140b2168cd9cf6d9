"""EGGROLL with Adam on B200 — the entry point of train/val/eggroll.py with the work in noise_b200.

Same command line, knobs, schedule and outputs as the reference script (argparse :171-179, data
shuffle :190-193, warmup-then-rebuild :214-219, linear warmdown :208-212, metrics.jsonl / result.json /
final.pt :221-247). The population forward, fitness shaping, Sigma f eps reconstruction and AdamW run
in the sm_100a kernels behind noise_b200's C ABI. FineWeb rows are read from --data-dir when present;
--synthetic substitutes seeded Zipf(1.1) rows of the same shape.

Launch: torchrun --standalone --nproc_per_node=8 train/val/eggroll.py [--synthetic]
"""
import argparse
import datetime
import json
import os
from pathlib import Path
import sys
import time

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from noise_b200.data import ROW, TRAIN_ROWS, VAL_ROWS, load_rows  # noqa: E402
from noise_b200.eggroll import BATCH, BETAS, CHUNK, LR, PAIRS, SEED, SIGMA, WARMDOWN, AdamW, Eggroll  # noqa: E402
from noise_b200.model import Weights  # noqa: E402
from noise_b200.population import evaluate  # noqa: E402

def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument('--data-dir', type=Path, default=Path('data'))
    parser.add_argument('--output', type=Path, default=Path('logs/eggroll'))
    parser.add_argument('--steps', type=int, help='Stop after this many updates (smoke tests).')
    parser.add_argument('--eval-every', type=int, default=0, help='Untimed validation every this many updates.')
    parser.add_argument('--pairs', type=int, default=PAIRS, help='Antithetic pairs per update.')
    parser.add_argument('--lr', type=float, default=LR, help='Adam learning rate.')
    parser.add_argument('--sigma', type=float, default=SIGMA, help='Perturbation scale.')
    parser.add_argument('--fitness', default='zscore', choices=['zscore', 'centered_rank'])
    parser.add_argument('--all-sequences', action='store_true', help='Every member evaluates all BATCH rows.')
    parser.add_argument('--synthetic', action='store_true', help='Zipf(1.1) rows when the FineWeb files are absent.')
    args = parser.parse_args()

    if not torch.cuda.is_available():
        parser.error('Training requires a CUDA GPU.')
    rank, world = int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1))
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', 0)))
    torch.cuda.set_device(device)
    if world > 1:
        torch.distributed.init_process_group('nccl', device_id=device, timeout=datetime.timedelta(minutes=10))
    members = 2 * args.pairs if args.all_sequences else max(2 * args.pairs, 2 * BATCH)
    if members % world or (not args.all_sequences and (2 * args.pairs) % (world * 2 * min(CHUNK, args.pairs))):
        parser.error('Each GPU must evaluate whole chunks of pairs.')

    training = load_rows(args.data_dir / 'train.pt', TRAIN_ROWS, args.synthetic, seed=1)
    training = training[torch.randperm(len(training), generator=torch.Generator().manual_seed(SEED + 1))]
    steps = min(len(training) // BATCH, args.steps or len(training))
    if rank == 0:
        if args.output.exists() and any(args.output.iterdir()):
            raise FileExistsError(f'Choose an empty output directory: {args.output}')
        args.output.mkdir(parents=True, exist_ok=True)
        (args.output / 'config.json').write_text(json.dumps(dict(
            script='train/val/eggroll.py', world=world, batch=BATCH, steps=steps, seed=SEED, pairs=args.pairs,
            sigma=args.sigma, lr=args.lr, betas=BETAS, warmdown=WARMDOWN, fitness=args.fitness,
            all_sequences=args.all_sequences, torch_version=torch.__version__, backend='noise_b200 sm_100a',
        ), indent=2) + '\n')

    def init():
        model = Weights(device, seed=SEED)
        optimizer = AdamW(model, lr=args.lr, betas=BETAS, eps=1e-8, weight_decay=0.0)
        es = Eggroll(model, args.pairs, rank, world, sigma=args.sigma, seed=SEED, fitness=args.fitness,
                     all_sequences=args.all_sequences, chunk=min(CHUNK, args.pairs))
        return model, optimizer, es

    def set_rate(optimizer, step):
        left = (steps - step + 1) / steps  # fraction of the epoch still ahead, this update included
        for group in optimizer.param_groups:
            group.setdefault('initial_lr', group['lr'])
            group['lr'] = group['initial_lr'] * min(1.0, left / WARMDOWN)

    # Untimed warmup on random tokens (module loading, workspace allocation), then rebuild from the
    # seed so the timed run starts exactly as if the warmup never happened.
    model, optimizer, es = init()
    noise = torch.randint(0, 4096, (BATCH, ROW), generator=torch.Generator().manual_seed(SEED)).to(device)
    es.step(noise[:, :-1].contiguous(), noise[:, 1:].contiguous(), optimizer, 0)
    model, optimizer, es = init()
    val = None
    if args.eval_every:
        val = load_rows(args.data_dir / 'val.pt', VAL_ROWS, args.synthetic, seed=2)

    if rank == 0:
        print(f'eggroll: {steps} steps, {args.pairs} pairs, sigma={args.sigma}, lr={args.lr}, GPUs={world}', flush=True)
    log = (args.output / 'metrics.jsonl').open('a') if rank == 0 else None
    torch.cuda.synchronize()
    start, paused, elapsed = time.perf_counter(), 0.0, 0.0
    step = 0
    for step in range(1, steps + 1):
        batch = training[(step - 1) * BATCH:step * BATCH].to(device)
        set_rate(optimizer, step)
        loss = es.step(batch[:, :-1].contiguous(), batch[:, 1:].contiguous(), optimizer, step)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - start - paused
        record = dict(step=step, population_loss=loss, train_seconds=round(elapsed, 2))
        if args.eval_every and step % args.eval_every == 0 and step < steps:
            pause = time.perf_counter()
            record['val_loss'] = evaluate(model, val)
            paused += time.perf_counter() - pause
        if rank == 0:
            print(json.dumps(record), flush=True)
            log.write(json.dumps(record) + '\n')

    state = model.state_dict()
    if val is None:
        val = load_rows(args.data_dir / 'val.pt', VAL_ROWS, args.synthetic, seed=2)
    val_loss = evaluate(model, val)
    if rank == 0:
        torch.save(state, args.output / 'final.pt')
        result = dict(val_loss=val_loss, train_seconds=round(elapsed, 2), steps=step, tokens=step * BATCH * 2048)
        (args.output / 'result.json').write_text(json.dumps(result, indent=2) + '\n')
        print(json.dumps(result), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == '__main__':
    main()
