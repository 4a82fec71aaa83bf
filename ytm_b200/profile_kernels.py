"""Launch every engine kernel once inside a profiler range (for ncu).

    python -m ytm_b200.profile_kernels
    ncu --clock-control none --profile-from-start off --section SpeedOfLight ... \
        python -m ytm_b200.profile_kernels

Warm-up work (training batches of the configuration-2 model, batch-1 training
of configuration 1 and 3 models, thermometer encoding) runs before
cudaProfilerStart; the profiled range then holds one training batch and one
inference pass of configuration 2 (65,536 samples), a transform, an encode,
two fused batch-1 samples each of configurations 1 and 3, a patch-wise
transform and a thermometer encode.

    python -m ytm_b200.profile_kernels --converged N

instead trains the configuration-2 model for N batches of 256 samples (no
profiler range) and then profiles one more batch (evaluation, thresholds,
feedback): the feedback of a converged model, where few (sample, class)
pairs are still active.
"""
import sys

import numpy as np
import torch

from ytm_b200 import synthetic
from ytm_b200.cutm import MultiClassTM
torch.cuda.set_device(0)
if len(sys.argv) > 2 and sys.argv[1] == '--converged':
    nb = int(sys.argv[2])
    X, y = synthetic.make('c2', 256 * (nb + 1))
    tm = MultiClassTM(seed=42, **synthetic.MODELS['c2'])
    lits = tm._encode_device(X); Y = torch.from_numpy(tm.encode_Y(y)).cuda(); e = tm.engine
    for i in range(nb + 1):
        if i == nb:
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
        cs = e.train_eval(lits[i*256:(i+1)*256], i*256, None, True); e.train_update(cs, Y[i*256:(i+1)*256], lits[i*256:(i+1)*256], i*256, None)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print('done', flush=True)
    sys.exit(0)
X, y = synthetic.make('c2', 256 * 5)
tm = MultiClassTM(seed=42, **synthetic.MODELS['c2'])
lits = tm._encode_device(X); Y = torch.from_numpy(tm.encode_Y(y)).cuda(); e = tm.engine
for i in range(4):
    cs = e.train_eval(lits[i*256:(i+1)*256], i*256, None, True); e.train_update(cs, Y[i*256:(i+1)*256], lits[i*256:(i+1)*256], i*256, None)
Xi, _ = synthetic.make('c2', 65536)
Xi_d = torch.from_numpy(Xi.view(np.int32)).cuda()
li = tm._encode_device(Xi)
X1, y1 = synthetic.make('c1', 600)
t1 = MultiClassTM(seed=1, **synthetic.MODELS['c1'])
l1 = t1._encode_device(X1); Y1 = torch.from_numpy(t1.encode_Y(y1)).cuda()
t1.engine.train_fit_b1(l1[:500], Y1[:500], 0, None)
X3, y3 = synthetic.make('c3', 300)
t3 = MultiClassTM(seed=1, **synthetic.MODELS['c3'])
l3 = t3._encode_device(X3); Y3 = torch.from_numpy(t3.encode_Y(y3)).cuda()
t3.engine.train_fit_b1(l3[:200], Y3[:200], 0, None)
kw4 = dict(synthetic.MODELS['c4']); kw4['number_of_clauses_per_class'] = 64
t4 = MultiClassTM(seed=1, **kw4)
img = torch.randint(0, 256, (2048, 32 * 32 * 3), dtype=torch.uint8, device='cuda')
t4.encode_thermometer(img, 8, on_device=True)
torch.cuda.synchronize()
torch.cuda.profiler.start()
i = 4
cs = e.train_eval(lits[i*256:(i+1)*256], i*256, None, True); e.train_update(cs, Y[i*256:(i+1)*256], lits[i*256:(i+1)*256], i*256, None)
e.infer(li)
e.transform(li[:4096])
e.encode(Xi_d)
t1.engine.train_fit_b1(l1[500:502], Y1[500:502], 500, None)
t3.engine.train_fit_b1(l3[200:202], Y3[200:202], 200, None)
t3.engine.transform_patchwise(l3[:16])
t4.encode_thermometer(img, 8, on_device=True)
torch.cuda.synchronize()
torch.cuda.profiler.stop()
print('done', flush=True)
