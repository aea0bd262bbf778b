"""Applications built on the framework: headless imaging, people counting / tracking, the
Thousand-Brains sequence memory, the cortical area models, an ONNX subset runtime, data sources
and the face-recognition descriptors.  CPU code unless a kernel is named."""
