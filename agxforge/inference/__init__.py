"""Model inference on the B200 (the reference's agxforge/inference module layout):

    models      each model's shapes
    catalog     which kernel form each role runs and its launch plan
    assemble    configure / build: the layer builder (weights, KV cache, decode graph on the device)
    execute     decode(): the decode loop and the reference's report keys
"""
