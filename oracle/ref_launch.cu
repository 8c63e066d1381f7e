// ref_launch.cu -- TEST/BASELINE INFRASTRUCTURE ONLY.
//
// Builds the reference's own CUDA kernels (crates/paged-kv-cuda/kernels/kernels.cu,
// included from the reference checkout at build time; nothing of it is copied
// here) into oracle/_ref/libref_kernels.so, with extern "C" launchers that use
// the launch shapes of the reference's CudaBackend:
//   reshape_and_cache: grid = num_tokens, block = 256, one launch per layer
//                      (crates/paged-kv-cuda/src/backend.rs:187-206)
//   copy_blocks:       grid = num_pairs * num_layers, block = 256 (backend.rs:275-290)
//   zero_block:        grid = num_layers, block = 256, one launch per block (backend.rs:304-317)
// Used to check the C oracle against the reference's device code and to time
// the reference kernels on B200 as the device-side "before" number.
#include <cuda_runtime.h>

#include REF_KERNELS_CU

extern "C" int ref_reshape_and_cache(const float *key, const float *value, float *key_cache,
                                     float *value_cache, const long long *slot_mapping,
                                     int num_tokens, int layer, int num_blocks, int block_size,
                                     int entry_elems, void *stream) {
    if (num_tokens <= 0) return 0;
    reshape_and_cache_kernel<<<num_tokens, 256, 0, (cudaStream_t)stream>>>(
        key, value, key_cache, value_cache, slot_mapping, layer, num_blocks, block_size, entry_elems);
    return (int)cudaGetLastError();
}

extern "C" int ref_copy_blocks(float *key_cache, float *value_cache, const long long *pairs,
                               int num_pairs, int num_layers, int num_blocks, int block_elems,
                               void *stream) {
    if (num_pairs <= 0) return 0;
    copy_blocks_kernel<<<num_pairs * num_layers, 256, 0, (cudaStream_t)stream>>>(
        key_cache, value_cache, pairs, num_pairs, num_layers, num_blocks, block_elems);
    return (int)cudaGetLastError();
}

extern "C" int ref_zero_block(float *key_cache, float *value_cache, int block, int num_layers,
                              int num_blocks, int block_elems, void *stream) {
    zero_block_kernel<<<num_layers, 256, 0, (cudaStream_t)stream>>>(
        key_cache, value_cache, block, num_layers, num_blocks, block_elems);
    return (int)cudaGetLastError();
}
