"""CPU oracle for the fused 2:4-sparse Conv/Linear + BN + LIF layer.

TEST INFRASTRUCTURE ONLY.  Nothing in the product path (``sparsesnn_b200``)
imports this package.  It is used by ``tests/``, by
``__graft_entry__.smoke()`` as the checker, and by ``bench.py``'s CPU
baseline / reference arm, which times it as a port of the reference's own
PyTorch CPU path.

Modules
-------
pack24     numpy restatement of the reference's 2:4 magnitude pruning
           (``sparse/pruning.py:28-76``) plus the packer that turns a pruned
           weight into compressed FP16 values and sparse-MMA metadata words.
lif_layer  numpy restatement of Conv2d + BatchNorm2d(eval) + multi-step LIF
           (``models/neurons.py:121-146,187-211``; ``models/layers.py:26-31``;
           ``models/sewresnet.py:50-66`` for the SEW residual add).
attention  numpy restatement of the Spikformer attention core + attention
           LIF (``models/spikformer.py:97,122-127``).
glue       numpy restatement of the Add -> LIF and MaxPool2d -> LIF patterns
           (``models/neurons.py``; torch ``MaxPool2d`` semantics).
sew_resnet torch-CPU port of the reference SEW-ResNet-18 forward
           (``models/sewresnet.py:123-210``) with the CIFAR stem, used as the
           timed CPU baseline and for end-to-end logit sanity checks.

Parity pin: ``tests/golden/make_golden.py`` imports the real reference
(``models.neurons``, ``sparse.pruning``) and writes seeded fixtures;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""
