//! # opencuda-cuda
//!
//! The B200 (sm_100a) backend of OpenCUDA.  [`CudaDevice`] implements
//! `opencuda_core::GpuDevice` (crates/opencuda-core/src/device.rs:88-132)
//! over the C ABI of libopencuda_cuda.so (include/opencuda_cuda.h):
//!
//! * `alloc` / `free` / `memcpy_*` / `synchronize` map one to one onto
//!   `oc_device_*`, with the CPU backend's contract (`alloc(0)` fails,
//!   unknown pointers are `GpuError::InvalidPtr`, oversize copies fail;
//!   crates/opencuda-cpu/src/lib.rs:85-151);
//! * `launch_kernel` routes by kernel name, as the Vulkan backend routes its
//!   SPIR-V entry points (crates/opencuda-vulkan/src/real.rs:868-887): the
//!   kernel's `Native` closure or SPIR-V bytes are not used, the library's
//!   own sm_100a kernel of that name runs instead (`sgemm_naive`, `matmul`,
//!   `quantize_symmetric`, `softmax`, `flash_attention`, `qgemm_w8`,
//!   `qgemm_w4`); other names fail with `GpuError::UnsupportedKernel`;
//! * `supports_spirv()` stays `false`, so `opencuda_blas::select_gemm_path`
//!   picks `GemmPath::CuBlas` for this NVIDIA device (blas:70-93) and
//!   `sgemm` runs the name-routed GEMM (rust/patches/opencuda-blas-cuda.patch).
//!
//! There is no CPU or Vulkan fallback inside this backend: a kernel it does
//! not know is an error.
//!
//! Status: written against the reference's interfaces but not compiled in
//! the repository that holds it (its image has no Rust toolchain); the
//! `extern "C"` declarations in `ffi.rs` are checked against the C header by
//! that repository's host tests.

pub mod ffi;

use std::ffi::{CStr, CString};
use std::os::raw::c_int;
use std::sync::Arc;

use opencuda_core::{
    CompiledKernel, DeviceInfo, DevicePtr, DeviceRegistry, GpuDevice, GpuError, GpuVendor, KernelArg,
    LaunchConfig, Result,
};

/// The calling thread's last library error message.
fn last_error() -> String {
    // SAFETY: oc_get_last_error returns a NUL-terminated thread-local string.
    unsafe { CStr::from_ptr(ffi::oc_get_last_error()) }
        .to_string_lossy()
        .into_owned()
}

/// Library status -> the reference's error types (GpuError::to_cuda_code,
/// crates/opencuda-core/src/error.rs:39-48, read backwards).
fn check(rc: c_int) -> Result<()> {
    match rc {
        ffi::OC_OK => Ok(()),
        ffi::OC_ERR_OUT_OF_MEMORY => Err(GpuError::OutOfMemory(0).into()),
        ffi::OC_ERR_NO_DEVICE => Err(GpuError::NoDevice.into()),
        ffi::OC_ERR_LAUNCH_FAILED => Err(GpuError::LaunchFailed(last_error()).into()),
        code => Err(anyhow::anyhow!("opencuda-cuda (status {code}): {}", last_error())),
    }
}

/// One CUDA device of the B200 backend.
pub struct CudaDevice {
    raw: *mut ffi::oc_device,
    info: DeviceInfo,
}

// The library locks each device object for the duration of a call, so one
// CudaDevice may be shared between threads (GpuDevice: Send + Sync).
unsafe impl Send for CudaDevice {}
unsafe impl Sync for CudaDevice {}

impl CudaDevice {
    /// Number of CUDA devices visible to this process.
    pub fn device_count() -> usize {
        let mut n: c_int = 0;
        // SAFETY: n is a valid out-pointer.
        if unsafe { ffi::oc_get_device_count(&mut n) } == ffi::OC_OK {
            n.max(0) as usize
        } else {
            0
        }
    }

    /// Opens CUDA device `ordinal`.
    pub fn new(ordinal: usize) -> Result<Arc<Self>> {
        let mut raw: *mut ffi::oc_device = std::ptr::null_mut();
        // SAFETY: raw is a valid out-pointer.
        check(unsafe { ffi::oc_device_open(ordinal as c_int, &mut raw) })?;
        // SAFETY: oc_device_info is plain old data; the library fills it.
        let mut info: ffi::oc_device_info = unsafe { std::mem::zeroed() };
        if let Err(e) = check(unsafe { ffi::oc_device_get_info(raw, &mut info) }) {
            unsafe { ffi::oc_device_close(raw) };
            return Err(e);
        }
        let name = unsafe { CStr::from_ptr(info.name.as_ptr()) }.to_string_lossy().into_owned();
        Ok(Arc::new(Self {
            raw,
            info: DeviceInfo {
                id: ordinal,
                vendor: GpuVendor::Nvidia {
                    compute_capability: (info.cc_major as u32, info.cc_minor as u32),
                },
                name,
                total_memory: info.total_memory,
                compute_units: info.compute_units,
            },
        }))
    }

    /// Registers every visible CUDA device (crates/opencuda-core/src/registry.rs).
    pub fn register_all(registry: &mut DeviceRegistry) -> Result<usize> {
        let n = Self::device_count();
        for i in 0..n {
            registry.register(Self::new(i)?);
        }
        Ok(n)
    }

    /// The library's device object, for the host-slice `oc_blas_*` and the
    /// device-resident `oc_gpt_*` entry points.
    pub fn raw(&self) -> *mut ffi::oc_device {
        self.raw
    }

    fn owned(&self, p: DevicePtr) -> Result<u64> {
        if p.device_id as usize != self.info.id {
            return Err(GpuError::InvalidPtr(p).into());
        }
        Ok(p.addr)
    }
}

impl Drop for CudaDevice {
    fn drop(&mut self) {
        // SAFETY: raw came from oc_device_open and is closed once.
        unsafe { ffi::oc_device_close(self.raw) };
    }
}

/// KernelArg (crates/opencuda-core/src/kernel.rs:88-100) -> oc_kernel_arg.
fn to_oc_arg(a: &KernelArg) -> ffi::oc_kernel_arg {
    match *a {
        KernelArg::Ptr(p) => ffi::oc_kernel_arg { kind: ffi::OC_ARG_PTR, v: ffi::oc_kernel_arg_value { ptr: p.addr } },
        KernelArg::U32(x) => ffi::oc_kernel_arg { kind: ffi::OC_ARG_U32, v: ffi::oc_kernel_arg_value { u32_: x } },
        KernelArg::I32(x) => ffi::oc_kernel_arg { kind: ffi::OC_ARG_I32, v: ffi::oc_kernel_arg_value { i32_: x } },
        KernelArg::F32(x) => ffi::oc_kernel_arg { kind: ffi::OC_ARG_F32, v: ffi::oc_kernel_arg_value { f32_: x } },
        KernelArg::Usize(x) => {
            ffi::oc_kernel_arg { kind: ffi::OC_ARG_USIZE, v: ffi::oc_kernel_arg_value { usize_: x as u64 } }
        }
    }
}

impl GpuDevice for CudaDevice {
    fn info(&self) -> &DeviceInfo {
        &self.info
    }

    fn alloc(&self, bytes: usize) -> Result<DevicePtr> {
        let mut addr = 0u64;
        // SAFETY: addr is a valid out-pointer.
        match unsafe { ffi::oc_device_alloc(self.raw, bytes, &mut addr) } {
            ffi::OC_OK => Ok(DevicePtr::new(addr, self.info.id as u32)),
            ffi::OC_ERR_OUT_OF_MEMORY => Err(GpuError::OutOfMemory(bytes).into()),
            rc => check(rc).map(|_| DevicePtr::new(0, self.info.id as u32)),
        }
    }

    fn free(&self, ptr: DevicePtr) -> Result<()> {
        let addr = self.owned(ptr)?;
        match unsafe { ffi::oc_device_free(self.raw, addr) } {
            ffi::OC_ERR_INVALID_VALUE => Err(GpuError::InvalidPtr(ptr).into()),
            rc => check(rc),
        }
    }

    fn memcpy_h2d(&self, dst: DevicePtr, src: &[u8]) -> Result<()> {
        let d = self.owned(dst)?;
        // SAFETY: src is a live host slice of src.len() bytes.
        check(unsafe { ffi::oc_device_memcpy_h2d(self.raw, d, src.as_ptr().cast(), src.len()) })
    }

    fn memcpy_d2h(&self, dst: &mut [u8], src: DevicePtr) -> Result<()> {
        let s = self.owned(src)?;
        // SAFETY: dst is a live host slice of dst.len() bytes.
        check(unsafe { ffi::oc_device_memcpy_d2h(self.raw, dst.as_mut_ptr().cast(), s, dst.len()) })
    }

    fn memcpy_d2d(&self, dst: DevicePtr, src: DevicePtr, bytes: usize) -> Result<()> {
        let (d, s) = (self.owned(dst)?, self.owned(src)?);
        check(unsafe { ffi::oc_device_memcpy_d2d(self.raw, d, s, bytes) })
    }

    fn launch_kernel(&self, kernel: &CompiledKernel, cfg: &LaunchConfig, args: &[KernelArg]) -> Result<()> {
        let name = CString::new(kernel.name.as_str())?;
        let a: Vec<ffi::oc_kernel_arg> = args.iter().map(to_oc_arg).collect();
        let c = ffi::oc_launch_config {
            grid: [cfg.grid.0, cfg.grid.1, cfg.grid.2],
            block: [cfg.block.0, cfg.block.1, cfg.block.2],
            shared_mem: cfg.shared_mem,
        };
        // SAFETY: name, c and a outlive the call; nargs is a.len().
        match unsafe { ffi::oc_device_launch(self.raw, name.as_ptr(), &c, a.as_ptr(), a.len()) } {
            ffi::OC_ERR_LAUNCH_FAILED if last_error().starts_with("kernel source not supported") => {
                Err(GpuError::UnsupportedKernel("kernel name not routed by the CUDA backend").into())
            }
            rc => check(rc),
        }
    }

    fn synchronize(&self) -> Result<()> {
        check(unsafe { ffi::oc_device_synchronize(self.raw) })
    }

    // supports_spirv() keeps the default `false`: select_gemm_path then picks
    // GemmPath::CuBlas for this device (blas:87-92).
}

/// The device-resident GPT decoder (GptModel with weights, KV cache and the
/// decode step on the GPU; crates/open-cuda-llm/src/lib.rs:635-942).
pub struct CudaGpt {
    raw: *mut ffi::oc_gpt,
    vocab: usize,
}

unsafe impl Send for CudaGpt {}

impl CudaGpt {
    /// A model for up to `max_batch` sequences with prompts of up to
    /// `max_prompt_len` tokens on CUDA device `ordinal`.
    pub fn new(ordinal: usize, cfg: ffi::oc_gpt_config, max_batch: usize, max_prompt_len: usize) -> Result<Self> {
        let mut raw: *mut ffi::oc_gpt = std::ptr::null_mut();
        check(unsafe {
            ffi::oc_gpt_create(ordinal as c_int, &cfg, max_batch as c_int, max_prompt_len as c_int, &mut raw)
        })?;
        Ok(Self { raw, vocab: cfg.vocab_size })
    }

    /// GptModel::load_random (llm:635-646): bit-identical weights, drawn on the GPU.
    pub fn load_random(&mut self, seed: u64) -> Result<()> {
        check(unsafe { ffi::oc_gpt_load_random(self.raw, seed) })
    }

    /// GptModel::enable_mla_kv_compression (llm:822-838): a d_c-dim latent
    /// K/V cache per head; 0 < d_c < head_dim.
    pub fn enable_mla_kv_compression(&mut self, d_c: usize, seed: u64) -> Result<()> {
        check(unsafe { ffi::oc_gpt_enable_mla(self.raw, d_c, seed) })
    }

    /// Uploads one tensor of a checkpoint (ids as in the C header).
    pub fn set_weight(&mut self, which: i32, layer: usize, values: &[f32]) -> Result<()> {
        check(unsafe { ffi::oc_gpt_set_weight(self.raw, which, layer as c_int, values.as_ptr(), values.len()) })
    }

    /// GptModel::generate (llm:910-929) for `prompts.len() / prompt_len`
    /// independent sequences; returns the generated ids per sequence.
    pub fn generate(&mut self, prompts: &[u32], prompt_len: usize, max_new: usize) -> Result<Vec<Vec<u32>>> {
        if prompt_len == 0 || prompts.len() % prompt_len != 0 {
            anyhow::bail!("open-cuda-llm: prompt_ids must not be empty");
        }
        let batch = prompts.len() / prompt_len;
        let mut out = vec![0u32; batch * max_new];
        let mut produced: c_int = 0;
        check(unsafe {
            ffi::oc_gpt_generate(
                self.raw,
                batch as c_int,
                prompts.as_ptr(),
                prompt_len as c_int,
                max_new as c_int,
                out.as_mut_ptr(),
                std::ptr::null_mut(),
                &mut produced,
            )
        })?;
        let n = produced.max(0) as usize;
        Ok(out.chunks(max_new).map(|row| row[..n].to_vec()).collect())
    }

    pub fn vocab_size(&self) -> usize {
        self.vocab
    }
}

impl Drop for CudaGpt {
    fn drop(&mut self) {
        unsafe { ffi::oc_gpt_destroy(self.raw) };
    }
}

#[cfg(test)]
mod tests {
    use super::*;

    // These run only on a machine with a CUDA device and the library built.
    fn device() -> Option<Arc<CudaDevice>> {
        if CudaDevice::device_count() == 0 {
            return None;
        }
        CudaDevice::new(0).ok()
    }

    #[test]
    fn alloc_zero_fails_and_copies_round_trip() {
        let Some(d) = device() else { return };
        assert!(d.alloc(0).is_err());
        let p = d.alloc(16).unwrap();
        let x: [u8; 16] = *b"0123456789abcdef";
        d.memcpy_h2d(p, &x).unwrap();
        let mut y = [0u8; 16];
        d.memcpy_d2h(&mut y, p).unwrap();
        assert_eq!(x, y);
        assert!(d.memcpy_h2d(p, &[0u8; 17]).is_err());
        d.free(p).unwrap();
        assert!(d.free(p).is_err());
    }

    #[test]
    fn sgemm_known_answer_through_blas() {
        // blas:1090-1133: [[1,2],[3,4]] . [[5,6],[7,8]] with alpha 2, beta 3 over ones
        let Some(d) = device() else { return };
        let mut c = vec![1.0f32; 4];
        opencuda_blas::sgemm(d.as_ref(), 2, 2, 2, 2.0, &[1.0, 2.0, 3.0, 4.0], &[5.0, 6.0, 7.0, 8.0], 3.0, &mut c, None)
            .unwrap();
        assert_eq!(c, vec![41.0, 47.0, 89.0, 103.0]);
    }

    #[test]
    fn unknown_kernel_is_unsupported() {
        let Some(d) = device() else { return };
        let k = CompiledKernel::native("vector_add", |_, _| {});
        let e = d.launch_kernel(&k, &LaunchConfig::linear(1, 1), &[]).unwrap_err();
        assert!(e.downcast_ref::<GpuError>().is_some());
    }
}
