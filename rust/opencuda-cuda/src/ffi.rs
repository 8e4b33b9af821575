//! Declarations of the C ABI in include/opencuda_cuda.h that this crate
//! calls.  Each mirrors its header prototype argument for argument (a host
//! test of the repository compares names and argument counts).  Pointers to
//! device memory travel as u64 (DevicePtr.addr); streams as *mut c_void.
#![allow(non_camel_case_types, dead_code)]

use std::os::raw::{c_char, c_int, c_void};

pub const OC_OK: c_int = 0;
pub const OC_ERR_INVALID_VALUE: c_int = 1;
pub const OC_ERR_OUT_OF_MEMORY: c_int = 2;
pub const OC_ERR_LAUNCH_FAILED: c_int = 8;
pub const OC_ERR_NO_DEVICE: c_int = 100;
pub const OC_ERR_NOT_SUPPORTED: c_int = 801;
pub const OC_ERR_TIMEOUT: c_int = 702;

pub const OC_ARG_PTR: c_int = 0;
pub const OC_ARG_U32: c_int = 1;
pub const OC_ARG_I32: c_int = 2;
pub const OC_ARG_F32: c_int = 3;
pub const OC_ARG_USIZE: c_int = 4;

#[repr(C)]
pub struct oc_device {
    _private: [u8; 0],
}

#[repr(C)]
pub struct oc_gpt {
    _private: [u8; 0],
}

#[repr(C)]
pub struct oc_device_info {
    pub ordinal: c_int,
    pub cc_major: c_int,
    pub cc_minor: c_int,
    pub total_memory: u64,
    pub compute_units: u32,
    pub name: [c_char; 256],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct oc_launch_config {
    pub grid: [u32; 3],
    pub block: [u32; 3],
    pub shared_mem: u32,
}

/// The value half of oc_kernel_arg: one 8-byte union member.
#[repr(C)]
#[derive(Clone, Copy)]
pub union oc_kernel_arg_value {
    pub ptr: u64,
    pub u32_: u32,
    pub i32_: i32,
    pub f32_: f32,
    pub usize_: u64,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct oc_kernel_arg {
    pub kind: c_int,
    pub v: oc_kernel_arg_value,
}

#[repr(C)]
#[derive(Clone, Copy, Default)]
pub struct oc_device_partition {
    pub device_id: usize,
    pub layer_start: usize,
    pub layer_end: usize,
}

/// GptConfig (crates/open-cuda-llm/src/lib.rs:45-69), as oc_gpt_config.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct oc_gpt_config {
    pub vocab_size: usize,
    pub hidden_size: usize,
    pub num_layers: usize,
    pub num_heads: usize,
    pub intermediate_size: usize,
    pub max_seq_len: usize,
    pub layer_norm_eps: f32,
}

extern "C" {
    // device object (GpuDevice)
    pub fn oc_get_device_count(count: *mut c_int) -> c_int;
    pub fn oc_device_open(ordinal: c_int, dev: *mut *mut oc_device) -> c_int;
    pub fn oc_device_close(dev: *mut oc_device) -> c_int;
    pub fn oc_device_get_info(dev: *const oc_device, info: *mut oc_device_info) -> c_int;
    pub fn oc_device_alloc(dev: *mut oc_device, bytes: usize, addr: *mut u64) -> c_int;
    pub fn oc_device_free(dev: *mut oc_device, addr: u64) -> c_int;
    pub fn oc_device_memcpy_h2d(dev: *mut oc_device, dst: u64, src: *const c_void, bytes: usize) -> c_int;
    pub fn oc_device_memcpy_d2h(dev: *mut oc_device, dst: *mut c_void, src: u64, bytes: usize) -> c_int;
    pub fn oc_device_memcpy_d2d(dev: *mut oc_device, dst: u64, src: u64, bytes: usize) -> c_int;
    pub fn oc_device_synchronize(dev: *mut oc_device) -> c_int;
    pub fn oc_device_launch(
        dev: *mut oc_device,
        kernel_name: *const c_char,
        cfg: *const oc_launch_config,
        args: *const oc_kernel_arg,
        nargs: usize,
    ) -> c_int;
    pub fn oc_device_stream(dev: *mut oc_device) -> *mut c_void;
    pub fn oc_get_last_error() -> *const c_char;

    // opencuda-multidev
    pub fn oc_partition_layers_by_memory(
        total_memory: *const u64,
        num_devices: usize,
        total_layers: usize,
        out: *mut oc_device_partition,
    ) -> c_int;
    pub fn oc_partition_layers(
        devices: *const *mut oc_device,
        num_devices: usize,
        total_layers: usize,
        out: *mut oc_device_partition,
    ) -> c_int;
    pub fn oc_transfer_between_devices(
        src: *mut oc_device,
        src_addr: u64,
        dst: *mut oc_device,
        dst_addr: u64,
        bytes: usize,
    ) -> c_int;

    // host-slice blas entry points (copy in, compute, copy out, synchronize)
    pub fn oc_blas_sgemm(
        dev: *mut oc_device,
        m: usize,
        k: usize,
        n: usize,
        alpha: f32,
        a: *const f32,
        b: *const f32,
        beta: f32,
        c: *mut f32,
    ) -> c_int;
    pub fn oc_blas_sdpa(
        dev: *mut oc_device,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        seq_len: usize,
        head_dim: usize,
        out: *mut f32,
    ) -> c_int;
    pub fn oc_blas_flash_attention(
        dev: *mut oc_device,
        q: *const f32,
        k: *const f32,
        v: *const f32,
        seq_len: usize,
        head_dim: usize,
        block_size: usize,
        out: *mut f32,
    ) -> c_int;
    pub fn oc_blas_mla_compress_kv(
        dev: *mut oc_device,
        seq_len: usize,
        d_h: usize,
        d_c: usize,
        kv: *const f32,
        down_proj: *const f32,
        latent: *mut f32,
    ) -> c_int;
    pub fn oc_blas_mla_decompress_kv(
        dev: *mut oc_device,
        seq_len: usize,
        d_c: usize,
        d_h: usize,
        latent: *const f32,
        up_proj: *const f32,
        out: *mut f32,
    ) -> c_int;
    pub fn oc_blas_quantize_int8(
        dev: *mut oc_device,
        input: *const f32,
        len: usize,
        group: usize,
        data: *mut i8,
        scales: *mut f32,
    ) -> c_int;
    pub fn oc_blas_quantize_int4(
        dev: *mut oc_device,
        input: *const f32,
        len: usize,
        group: usize,
        data: *mut u8,
        scales: *mut f32,
    ) -> c_int;
    pub fn oc_blas_qgemm_w8(
        dev: *mut oc_device,
        m: usize,
        n: usize,
        k: usize,
        a: *const f32,
        wq: *const i8,
        w_scales: *const f32,
        bias: *const f32,
        y: *mut f32,
    ) -> c_int;
    pub fn oc_blas_qgemm_w4(
        dev: *mut oc_device,
        m: usize,
        n: usize,
        k: usize,
        group: usize,
        a: *const f32,
        wq: *const u8,
        w_scales: *const f32,
        bias: *const f32,
        y: *mut f32,
    ) -> c_int;
    pub fn oc_blas_qgemm_w8a8(
        dev: *mut oc_device,
        m: usize,
        n: usize,
        k: usize,
        a: *const f32,
        wq: *const i8,
        w_scales: *const f32,
        bias: *const f32,
        y: *mut f32,
    ) -> c_int;
    pub fn oc_blas_qgemm_w4a8(
        dev: *mut oc_device,
        m: usize,
        n: usize,
        k: usize,
        group: usize,
        a: *const f32,
        wq: *const u8,
        w_scales: *const f32,
        bias: *const f32,
        y: *mut f32,
    ) -> c_int;

    // device-resident GPT decoder (GptModel)
    pub fn oc_gpt_create(
        ordinal: c_int,
        config: *const oc_gpt_config,
        max_batch: c_int,
        max_prompt_len: c_int,
        model: *mut *mut oc_gpt,
    ) -> c_int;
    pub fn oc_gpt_destroy(model: *mut oc_gpt) -> c_int;
    pub fn oc_gpt_load_random(model: *mut oc_gpt, seed: u64) -> c_int;
    pub fn oc_gpt_enable_mla(model: *mut oc_gpt, d_c: usize, seed: u64) -> c_int;
    pub fn oc_gpt_set_weight(model: *mut oc_gpt, which: c_int, layer: c_int, values: *const f32, len: usize) -> c_int;
    pub fn oc_gpt_generate(
        model: *mut oc_gpt,
        batch: c_int,
        prompt_ids: *const u32,
        prompt_len: c_int,
        max_new_tokens: c_int,
        out_tokens: *mut u32,
        out_logits: *mut f32,
        produced: *mut c_int,
    ) -> c_int;
}
