"""carbon_rec: Carbon-OCR's line recognition (crop, the rec-latin recognizer, greedy CTC)
rebuilt for B200 (sm_100a) behind a C ABI (include/carbon_rec.h).

Modules:
  native   ctypes binding of the C ABI and RecDevice, the recognizer backend a pipeline drives
  build    compiles csrc/*.cu into libcarbon_rec.so (sm_100a) in-tree
  netdef   an ONNX recognizer compiled into the layer list and model blob the library runs
  model    rec-latin's shapes, random-init weights, FP32 and INT8 Q/DQ ONNX files
  onnx_pb  the ONNX protobuf reader and writer
  synth    seeded synthetic pages, boxes and crops of the benchmark configurations
"""
