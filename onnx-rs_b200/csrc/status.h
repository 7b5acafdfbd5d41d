// Status codes shared by host code, device code and the public C ABI.
#pragma once

// Each code maps 1:1 onto a variant of the reference's crate::error::Error
// (src/error.rs:19-66).
#define ONNXB200_OK 0
#define ONNXB200_ERR_VALIDATION 1         /* Error::ValidationError */
#define ONNXB200_ERR_EXECUTION 2          /* Error::ExecutionError (CUDA error) */
#define ONNXB200_ERR_UNSUPPORTED 3        /* Error::UnsupportedFeature */
#define ONNXB200_ERR_TIMEOUT 4            /* Error::OperationTimeout (bounded wait expired) */
#define ONNXB200_ERR_RESOURCE_EXHAUSTED 5 /* Error::ResourceExhausted (allocation / workspace) */
#define ONNXB200_ERR_INVALID_GRAPH 6      /* Error::InvalidGraph */
#define ONNXB200_ERR_INVALID_OPERATOR 7   /* Error::InvalidOperator (op not in registry) */
#define ONNXB200_ERR_CANCELLED 8          /* Error::ExecutionCancelled */
#define ONNXB200_ERR_INVALID_ARGUMENT 9   /* null handle / pointer (no reference variant) */
#define ONNXB200_ERR_IO 10                /* Error::IoError / Error::ModelLoadError */
#define ONNXB200_ERR_PROTOBUF 11          /* Error::ProtobufError (malformed model bytes) */
#define ONNXB200_ERR_INVALID_MODEL 12     /* Error::InvalidModel / Error::MissingField */
