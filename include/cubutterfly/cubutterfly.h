/*
 * cubutterfly.h -- public C ABI of cubutterfly_b200.
 *
 * Drop-in replacement for the reference's include/cubutterfly/cubutterfly.h:
 * every entry point, enum value and struct layout below is the one a caller of
 * that header binds to (reference include/cubutterfly/cubutterfly.h:18-318).
 * Each declaration cites the reference line it replaces.  The implementation
 * (cubutterfly_b200/csrc) is new: a C++ planner with a B200 hardware profile
 * and hand-written sm_100a kernels.  Requests outside the executable scope
 * return CUBUTTERFLY_STATUS_NOT_SUPPORTED with a reason in
 * cubutterflyGetLastErrorString(), as the reference does for its own gaps.
 */
#ifndef CUBUTTERFLY_B200_CUBUTTERFLY_H
#define CUBUTTERFLY_B200_CUBUTTERFLY_H

#include <cuda_runtime_api.h>
#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#define CUBUTTERFLYAPI __declspec(dllimport)
#else
#define CUBUTTERFLYAPI __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Version reported by cubutterflyGetVersion (reference cubutterfly.h:18-20). */
#define CUBUTTERFLY_VERSION_MAJOR 0
#define CUBUTTERFLY_VERSION_MINOR 9
#define CUBUTTERFLY_VERSION_PATCH 3
#define CUBUTTERFLY_MAX_EXECUTION_RANK 8

/* Logical index order of one axis (reference :26-29).  A bit-reversed axis
 * stores logical coordinate i at reverse_bits(i, log2(extent)). */
typedef enum cubutterflyLogicalOrder {
    CUBUTTERFLY_ORDER_NATURAL = 0,
    CUBUTTERFLY_ORDER_BIT_REVERSED = 1
} cubutterflyLogicalOrder_t;

/* Opaque objects (reference :31-33). */
typedef struct cubutterflyHandle* cubutterflyHandle_t;
typedef struct cubutterflyDescriptor* cubutterflyDescriptor_t;
typedef struct cubutterflyPlan* cubutterflyPlan_t;

/* Status codes (reference :35-44). */
typedef enum cubutterflyStatus {
    CUBUTTERFLY_STATUS_SUCCESS = 0,
    CUBUTTERFLY_STATUS_INVALID_VALUE = 1,
    CUBUTTERFLY_STATUS_INVALID_TYPE = 2,
    CUBUTTERFLY_STATUS_NOT_SUPPORTED = 3,
    CUBUTTERFLY_STATUS_ALLOC_FAILED = 4,
    CUBUTTERFLY_STATUS_CUDA_ERROR = 5,
    CUBUTTERFLY_STATUS_BACKEND_ERROR = 6,
    CUBUTTERFLY_STATUS_INTERNAL_ERROR = 7
} cubutterflyStatus_t;

/* Butterfly operator family (reference :46-53). */
typedef enum cubutterflyOperator {
    CUBUTTERFLY_OPERATOR_FFT = 0,
    CUBUTTERFLY_OPERATOR_NTT = 1,
    CUBUTTERFLY_OPERATOR_FWHT = 2,
    CUBUTTERFLY_OPERATOR_SUBSET_ZETA = 3,
    CUBUTTERFLY_OPERATOR_SUPERSET_ZETA = 4,
    CUBUTTERFLY_OPERATOR_STRUCTURED_2X2 = 5
} cubutterflyOperator_t;

/* Storage element type (reference :55-66). */
typedef enum cubutterflyDataType {
    CUBUTTERFLY_DATA_FP16 = 0,
    CUBUTTERFLY_DATA_BF16 = 1,
    CUBUTTERFLY_DATA_FP32 = 2,
    CUBUTTERFLY_DATA_FP64 = 3,
    CUBUTTERFLY_DATA_COMPLEX_FP16 = 4,
    CUBUTTERFLY_DATA_COMPLEX_BF16 = 5,
    CUBUTTERFLY_DATA_COMPLEX_FP32 = 6,
    CUBUTTERFLY_DATA_COMPLEX_FP64 = 7,
    CUBUTTERFLY_DATA_UINT32 = 8,
    CUBUTTERFLY_DATA_UINT64 = 9
} cubutterflyDataType_t;

/* Arithmetic domain (reference :68-74). */
typedef enum cubutterflyComputeType {
    CUBUTTERFLY_COMPUTE_NATIVE = 0,
    CUBUTTERFLY_COMPUTE_FP32 = 1,
    CUBUTTERFLY_COMPUTE_FP64 = 2,
    CUBUTTERFLY_COMPUTE_UINT32 = 3,
    CUBUTTERFLY_COMPUTE_UINT64 = 4
} cubutterflyComputeType_t;

/* reference :76-79 */
typedef enum cubutterflyDirection {
    CUBUTTERFLY_DIRECTION_FORWARD = 0,
    CUBUTTERFLY_DIRECTION_INVERSE = 1
} cubutterflyDirection_t;

/* reference :81-84 */
typedef enum cubutterflyPlacement {
    CUBUTTERFLY_PLACEMENT_OUT_OF_PLACE = 0,
    CUBUTTERFLY_PLACEMENT_IN_PLACE = 1
} cubutterflyPlacement_t;

/* reference :88-91 */
typedef enum cubutterflyArithmeticPolicy {
    CUBUTTERFLY_ARITHMETIC_STRICT = 0,
    CUBUTTERFLY_ARITHMETIC_ALLOW_FP16_MMA = 1
} cubutterflyArithmeticPolicy_t;

/* STAGE_STORAGE rounds to the storage type after every stage; FINAL_STORAGE
 * keeps the compute type until the output scale and one final narrowing
 * (reference :86-96). */
typedef enum cubutterflyOutputRounding {
    CUBUTTERFLY_ROUNDING_STAGE_STORAGE = 0,
    CUBUTTERFLY_ROUNDING_FINAL_STORAGE = 1
} cubutterflyOutputRounding_t;

/* reference :98-101 */
typedef enum cubutterflyLengthMode {
    CUBUTTERFLY_LENGTH_STANDARD = 0,
    CUBUTTERFLY_LENGTH_ZERO_EXTENDED_EMBEDDING = 1
} cubutterflyLengthMode_t;

/* reference :106-110 */
typedef enum cubutterflyExecutionMode {
    CUBUTTERFLY_EXECUTION_AUTO = 0,
    CUBUTTERFLY_EXECUTION_XD = 1,
    CUBUTTERFLY_EXECUTION_COMPOSITE = 2
} cubutterflyExecutionMode_t;

/* reference :115-119 */
typedef enum cubutterflyFftTransformType {
    CUBUTTERFLY_FFT_C2C = 0,
    CUBUTTERFLY_FFT_R2C = 1,
    CUBUTTERFLY_FFT_C2R = 2
} cubutterflyFftTransformType_t;

/* reference :121-127 */
typedef enum cubutterflyNttLayout {
    CUBUTTERFLY_NTT_LAYOUT_NATURAL = 0,
    CUBUTTERFLY_NTT_LAYOUT_APPT_STATIC = 1,
    CUBUTTERFLY_NTT_LAYOUT_BIT_REVERSED = 2
} cubutterflyNttLayout_t;

/* reference :129-137 (layout and size are part of the ABI) */
typedef struct cubutterflyNttLayoutInfo {
    uint32_t log_n;
    uint32_t stage_count;
    uint32_t stage_partition[3];
    uint32_t fragment_width;
    uint32_t bank_bits;
    int xor_permutation;
    char compatibility_id[64];
} cubutterflyNttLayoutInfo_t;

/* reference :139-143 */
typedef enum cubutterflyAlgorithmPolicy {
    CUBUTTERFLY_ALGORITHM_DEFAULT = 0,
    CUBUTTERFLY_ALGORITHM_MEASURE = 1,
    CUBUTTERFLY_ALGORITHM_EXPLICIT = 2
} cubutterflyAlgorithmPolicy_t;

/* reference :145-153 */
typedef enum cubutterflySelectionSource {
    CUBUTTERFLY_SELECTION_MEASURED_TABLE = 0,
    CUBUTTERFLY_SELECTION_USER_CACHE = 1,
    CUBUTTERFLY_SELECTION_RUNTIME_MEASURED = 2,
    CUBUTTERFLY_SELECTION_STATIC_MODEL = 3,
    CUBUTTERFLY_SELECTION_EXPLICIT = 4,
    CUBUTTERFLY_SELECTION_UNMEASURED_FALLBACK = 5
} cubutterflySelectionSource_t;

/* reference :155-159 */
typedef enum cubutterflyLogLevel {
    CUBUTTERFLY_LOG_INFO = 0,
    CUBUTTERFLY_LOG_WARNING = 1,
    CUBUTTERFLY_LOG_ERROR = 2
} cubutterflyLogLevel_t;

/* reference :161-166 (four doubles, row major) */
typedef struct cubutterflyMatrix2x2 {
    double m00;
    double m01;
    double m10;
    double m11;
} cubutterflyMatrix2x2_t;

/* reference :168-171 */
typedef void (*cubutterflyLogCallback_t)(cubutterflyLogLevel_t level, const char* event, const char* message,
                                         void* user_data);

/* ---- status, errors, version (reference :173-177) ---------------------- */
CUBUTTERFLYAPI const char* cubutterflyGetStatusString(cubutterflyStatus_t status);
/* Detailed error of the calling thread's last protected call; it stays valid
 * until that thread's next protected call and reading it does not clear it. */
CUBUTTERFLYAPI const char* cubutterflyGetLastErrorString(void);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyGetVersion(int* major, int* minor, int* patch);

/* ---- handle: stream, log callback, plan cache (reference :179-186) ------ */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyCreate(cubutterflyHandle_t* handle);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDestroy(cubutterflyHandle_t handle);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetStream(cubutterflyHandle_t handle, cudaStream_t stream);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyGetStream(cubutterflyHandle_t handle, cudaStream_t* stream);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetLogCallback(cubutterflyHandle_t handle,
                                                            cubutterflyLogCallback_t callback, void* user_data);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetCachePath(cubutterflyHandle_t handle, const char* path);

/* ---- legacy real-FFT adapters (reference :188-194); return nonzero on
 * failure.  Real FFTs are outside this build's scope: both return
 * CUBUTTERFLY_STATUS_NOT_SUPPORTED. */
CUBUTTERFLYAPI int cubutterflyPackRealFp32(const float* input, void* output, size_t elements, float scale,
                                           uint64_t stream);
CUBUTTERFLYAPI int cubutterflyExpandHermitianFp32(const void* half, void* full, uint32_t height, uint32_t width,
                                                  size_t batch, uint64_t stream);

/* ---- descriptor (reference :196-276) ------------------------------------ */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyCreateDescriptor(cubutterflyDescriptor_t* descriptor);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDestroyDescriptor(cubutterflyDescriptor_t descriptor);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetOperator(cubutterflyDescriptor_t descriptor,
                                                         cubutterflyOperator_t op);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetDataType(cubutterflyDescriptor_t descriptor,
                                                         cubutterflyDataType_t storage,
                                                         cubutterflyComputeType_t compute);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetShape(cubutterflyDescriptor_t descriptor, uint32_t rank,
                                                      const size_t* extents, size_t batch);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetExecutionMode(cubutterflyDescriptor_t descriptor,
                                                              cubutterflyExecutionMode_t mode);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetFftTransformType(cubutterflyDescriptor_t descriptor,
                                                                 cubutterflyFftTransformType_t type);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetFftOutputScale(cubutterflyDescriptor_t descriptor, double scale);
/* Output scale applied before the final narrowing (default 1). */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetOutputScale(cubutterflyDescriptor_t descriptor, double scale);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetArithmeticPolicy(cubutterflyDescriptor_t descriptor,
                                                                 cubutterflyArithmeticPolicy_t policy);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetOutputRounding(cubutterflyDescriptor_t descriptor,
                                                               cubutterflyOutputRounding_t rounding);
/* NULL selects packed axis strides for that side; a zero batch stride selects
 * the packed span. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetStrides(cubutterflyDescriptor_t descriptor,
                                                        const size_t* input_strides, size_t input_batch_stride,
                                                        const size_t* output_strides, size_t output_batch_stride);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetLogicalOrders(cubutterflyDescriptor_t descriptor,
                                                              const cubutterflyLogicalOrder_t* input_orders,
                                                              const cubutterflyLogicalOrder_t* output_orders);
/* CPU-only validation and canonical JSON.  String queries take a NULL buffer
 * to return the size including the trailing NUL. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDescriptorValidate(cubutterflyDescriptor_t descriptor);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDescriptorGetJson(cubutterflyDescriptor_t descriptor, char* json,
                                                               size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDescriptorSetJson(cubutterflyDescriptor_t descriptor,
                                                               const char* json);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDescriptorGetCapabilities(cubutterflyDescriptor_t descriptor,
                                                                       char* json, size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetDirection(cubutterflyDescriptor_t descriptor,
                                                          cubutterflyDirection_t direction, int normalize_inverse);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetPlacement(cubutterflyDescriptor_t descriptor,
                                                          cubutterflyPlacement_t placement);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetLengthMode(cubutterflyDescriptor_t descriptor,
                                                           cubutterflyLengthMode_t mode);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetAlgorithmPolicy(cubutterflyDescriptor_t descriptor,
                                                                cubutterflyAlgorithmPolicy_t policy,
                                                                const char* explicit_algorithm);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetModulus(cubutterflyDescriptor_t descriptor, uint64_t modulus,
                                                        uint32_t word_bits);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetNttLayouts(cubutterflyDescriptor_t descriptor,
                                                           cubutterflyNttLayout_t input_layout,
                                                           cubutterflyNttLayout_t output_layout);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflySetStageMatrices(cubutterflyDescriptor_t descriptor, uint32_t axis,
                                                              const cubutterflyMatrix2x2_t* matrices,
                                                              size_t count);

/* ---- plans (reference :278-318) ----------------------------------------- */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyCreatePlan(cubutterflyHandle_t handle,
                                                        cubutterflyDescriptor_t descriptor,
                                                        cubutterflyPlan_t* plan);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyDestroyPlan(cubutterflyPlan_t plan);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetDescriptorJson(cubutterflyPlan_t plan, char* json,
                                                                   size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetWorkspaceSize(cubutterflyPlan_t plan, size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetInputSize(cubutterflyPlan_t plan, size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetOutputSize(cubutterflyPlan_t plan, size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetPhysicalExtents(cubutterflyPlan_t plan, size_t* extents,
                                                                    uint32_t capacity);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetSelectionSource(cubutterflyPlan_t plan,
                                                                    cubutterflySelectionSource_t* source);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetAlgorithmName(cubutterflyPlan_t plan, char* name,
                                                                  size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetSelectionReason(cubutterflyPlan_t plan, char* reason,
                                                                    size_t* bytes);
/* Full mapping; a mapping JSON can be passed back through the EXPLICIT policy. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetMappingJson(cubutterflyPlan_t plan, char* json,
                                                                size_t* bytes);
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanGetNttLayoutInfo(cubutterflyPlan_t plan,
                                                                  cubutterflyNttLayoutInfo_t* info);
/* Caller-owned workspace: at least PlanGetWorkspaceSize bytes, 16-byte aligned. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyPlanSetWorkspace(cubutterflyPlan_t plan, void* workspace,
                                                              size_t bytes);
/* Asynchronous on the handle's stream; allocates nothing.  In-place plans
 * require input == output, out-of-place plans distinct pointers. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyExecute(cubutterflyHandle_t handle, cubutterflyPlan_t plan,
                                                     const void* input, void* output);
/* Reused-plan submission; the first call and any call after a stream change
 * take the cubutterflyExecute path. */
CUBUTTERFLYAPI cubutterflyStatus_t cubutterflyExecuteSteady(cubutterflyHandle_t handle, cubutterflyPlan_t plan,
                                                           const void* input, void* output);

#ifdef __cplusplus
}
#endif

#endif /* CUBUTTERFLY_B200_CUBUTTERFLY_H */
