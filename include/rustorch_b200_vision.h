/*
 * rustorch_b200_vision.h — C entry points for the ResNet-18 inference model
 * built from the backend's ops (rustorch::vision::ResNet18 in
 * include/rustorch_b200.hpp).  The reference's rustorch-vision ResNet is an
 * empty placeholder (rustorch-vision/src/models.rs:1); this model is composed
 * from the reference's own ops: conv2d + bias + relu, max_pool2d, residual
 * add, global average pool and Linear.
 */
#ifndef RUSTORCH_B200_VISION_H
#define RUSTORCH_B200_VISION_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Builds the model on `device` with seeded weights: conv weights
 * Kaiming-normal (std sqrt(2/fan_in)) from (seed, conv index), BatchNorm
 * folded with gamma 1, beta 0, mean 0, var 1, eps 1e-5; fc weight/bias
 * U(-1/sqrt(512), 1/sqrt(512)) from (seed, 100/101). */
int rtb_resnet18_create(int device, uint64_t seed, int precision, void** handle);
int rtb_resnet18_destroy(void* handle);
/* logits [batch, 1000] = ResNet-18(x [batch, 3, 224, 224] NCHW); both device
 * pointers on the model's device; ordered on `stream`. */
int rtb_resnet18_forward(void* handle, int64_t batch, const float* x_nchw, float* logits,
                         void* stream);
/* Parameters: 20 x (conv weight [Co,Ci,k,k], folded bias [Co]), fc.weight,
 * fc.bias.  Copies parameter `index` to host_out (may be NULL) and its shape
 * (padded with 1s) to shape4. */
int64_t rtb_resnet18_num_params(void* handle);
int rtb_resnet18_get_param(void* handle, int64_t index, float* host_out, int64_t* shape4);
int64_t rtb_resnet18_flops_per_image(void* handle);

#ifdef __cplusplus
}
#endif
#endif /* RUSTORCH_B200_VISION_H */
