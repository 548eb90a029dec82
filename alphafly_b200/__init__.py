"""alphafly_b200: alpha-fly's connectome recurrence on B200.

Modules mirror the reference's: ``brain`` (ConnectomeRNN, LightCone; chessfly/brain.py), ``model``
(FlyChessNet, RunningNorm, Evaluator; chessfly/model.py), ``train`` (train_step; chessfly/train.py),
``connectome`` and ``encoding``; plus ``webmodel`` (the browser model format), ``synth`` (synthetic graphs
and inputs) and ``_lib`` (the ctypes binding of libafb.so, the CUDA library).
"""
